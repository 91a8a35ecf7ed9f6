"""Router R1..R5 on the device vs the declared-order C restatement: bit-exact."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(cuda, x, xdtype, wg_bits, bias=None):
    import torch
    from b200moe import _abi
    T = x.shape[0]
    xt = torch.from_numpy(x).to(cuda)
    wg = torch.from_numpy(wg_bits.view(np.int16)).view(torch.bfloat16).to(cuda)
    bt = None if bias is None else torch.from_numpy(bias).to(cuda)
    logits = torch.empty((T, 256), dtype=torch.int16, device=cuda)
    ids = torch.empty((T, 8), dtype=torch.int32, device=cuda)
    wf = torch.empty((T, 8), dtype=torch.float32, device=cuda)
    wb = torch.empty((T, 8), dtype=torch.int16, device=cuda)
    _abi.router(xt, xdtype, T, wg, bt, logits, ids, wf, wb)
    torch.cuda.synchronize()
    return dict(logits=logits.cpu().numpy().view(np.uint16), ids=ids.cpu().numpy(), w_f32=wf.cpu().numpy(),
                w_bf16=wb.cpu().numpy().view(np.uint16))


def _check(got, ref):
    assert (got["logits"] == ref["logits"]).all()
    assert (got["ids"] == ref["ids"]).all()
    assert (got["w_f32"].view(np.uint32) == ref["w_f32"].view(np.uint32)).all()
    assert (got["w_bf16"] == ref["w_bf16"]).all()


@pytest.mark.parametrize("T", [1, 7, 8, 9, 64])
def test_router_bf16_tokens(cuda, T):
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import _abi, synth
    x = synth.tokens(0, T, stream=3)
    wg = synth.router_w(0, 0)
    got = _run(cuda, x.view(np.int16), _abi.BF16, wg)
    _check(got, OM.router(bf16_bits_to_f32(x), wg))


def test_router_f32_tokens_and_bias(cuda):
    """f32 activations (inexact products: fused multiply-add order matters) + Zipf bias."""
    from oracle import moe as OM
    from b200moe import _abi, synth
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((33, 2048)) * 0.7).astype(np.float32)
    wg = synth.router_w(2, 4)
    bias = synth.zipf_bias(2, 4)
    got = _run(cuda, x, _abi.F32, wg, bias)
    _check(got, OM.router(x, wg, bias))


def test_router_exact_ties_lowest_index(cuda):
    """Duplicated router rows give exactly equal logits: the tie goes to the lower index."""
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import _abi, synth
    wg = synth.router_w(0, 1).copy()
    x = synth.tokens(0, 16, stream=4)
    ref0 = OM.router(bf16_bits_to_f32(x), wg)
    for t in range(16):             # copy the rank-1 expert's row onto a higher index
        e = ref0["ids"][t][0]
        wg[(e + 97) % 256] = wg[e]
    ref = OM.router(bf16_bits_to_f32(x), wg)
    got = _run(cuda, x.view(np.int16), _abi.BF16, wg)
    _check(got, ref)
    ntie = sum(1 for t in range(16) for k in range(7)
               if ref["logits"][t][ref["ids"][t][k]] == ref["logits"][t][ref["ids"][t][k + 1]])
    assert ntie >= 8
