"""The grouped small-batch decode path (csrc/grouped.cu): 2..16 tokens of a Q4_K layer, every
distinct expert's rows read once and applied to all its tokens (two tokens per int8 tensor-core
MMA), then the ordered combine.

Parity bar as for every decode path (tests/test_gpu_decode.py): routing ids bit-exact against
the declared-order C restatement; the f32 block output against the f64 restatement of
engine/m3_forward.py:430-476 (fed the same ids) within rel-L2 1e-5 and max-abs / max|ref| 1e-5.
The Zipf logit bias (config 2's routing law) makes tokens share experts heavily, so experts
with many tokens (odd and even counts) occur. Copies of one token in a batch must get the same
bits, whatever their position or partner in a token pair; repeated calls the same bits.
"""
import numpy as np
import pytest

from conftest import host_layer

pytestmark = pytest.mark.gpu
REL_L2, MAX_ABS_NORM = 1e-5, 1e-5


@pytest.fixture(scope="module")
def zipf_layer(cuda):
    from b200moe.engine import DeviceLayer
    return DeviceLayer.synthetic(2, 0, cuda, bias=True)


def _tokens(T, stream, cuda):
    import torch
    from b200moe import synth
    xb = synth.tokens(2, T, stream=stream)
    return xb, torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)


@pytest.mark.parametrize("T", [2, 7, 16])
def test_grouped_vs_oracle(cuda, zipf_layer, T):
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe
    xb, x = _tokens(T, 40 + T, cuda)
    out, info = moe.moe_block(x, zipf_layer, path="decode")
    torch.cuda.synchronize()
    ids = info["ids"].cpu().numpy().reshape(T, 8)
    Lh = host_layer(2, 0, bias=True)
    xf = bf16_bits_to_f32(xb)
    r = OM.router(xf, Lh.wg, Lh.bias)
    assert (ids == r["ids"]).all()
    counts = np.bincount(ids.reshape(-1), minlength=256)
    if T >= 7:
        assert counts.max() >= 3          # experts shared by several tokens
    ref = OM.moe_block_f64(xf, Lh, ids, r["w_bf16"])["out"]
    c = OM.compare(out.reshape(T, 2048).cpu().numpy(), ref)
    print("grouped T=%d: distinct experts %d, most tokens on one expert %d, rel-L2 %.3e, max-abs/max %.3e"
          % (T, int((counts > 0).sum()), int(counts.max()), c["rel_l2"], c["max_abs_norm"]))
    assert c["rel_l2"] < REL_L2 and c["max_abs_norm"] < MAX_ABS_NORM, c


def test_grouped_copies_and_repeats_bit_identical(cuda, zipf_layer):
    """16 tokens: 5 distinct ones, each repeated at several positions (so copies sit in the
    first and the second column group of different token pairs); two calls."""
    import torch
    from b200moe import moe
    _, x5 = _tokens(5, 60, cuda)
    order = [0, 1, 2, 0, 3, 4, 1, 0, 2, 3, 4, 4, 1, 2, 3, 0]
    x = x5[order]
    a, ia = moe.moe_block(x, zipf_layer, path="decode")
    b, ib = moe.moe_block(x, zipf_layer, path="decode")
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(ia["ids"], ib["ids"])
    assert torch.isfinite(a).all()
    for u in range(5):
        rows = [i for i, o in enumerate(order) if o == u]
        for i in rows[1:]:
            assert torch.equal(a[rows[0]], a[i]), (u, i)
            assert torch.equal(ia["ids"][rows[0]], ia["ids"][i])
