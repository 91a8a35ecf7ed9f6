"""The combine order, pinned bit for bit (the f32 output bars cannot see it): through the stage
API on the prefill path, ``routed_sum`` must equal the f32 fold, in ascending expert id, of each
slot's ``expert_raw`` times its bf16 routing weight -- product and sum rounded separately, as
engine/m3_forward.py:452,464-465 adds the experts -- and must differ from the rank-order fold
somewhere (so the check can tell the two apart)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _fold(raw, w, order):
    acc = np.zeros(raw.shape[-1], np.float32)
    for k in order:
        acc = (acc + (raw[k] * np.float32(w[k])).astype(np.float32)).astype(np.float32)
    return acc


def test_routed_sum_is_the_ascending_id_fold(cuda):
    import torch
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    from b200moe.engine import DeviceLayer
    L = DeviceLayer.synthetic(0, 0, cuda)
    T = 16
    xb = synth.tokens(0, T, stream=77)
    g = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    st = moe.moe_block_stages(g, L)
    torch.cuda.synchronize()
    raw = st["expert_raw"].cpu().numpy()
    ids = st["topk_ids"].cpu().numpy()
    w = bf16_bits_to_f32(st["topk_weights"].view(torch.int16).cpu().numpy().view(np.uint16))
    got = st["routed_sum"].cpu().numpy()
    rank_differs = 0
    for t in range(T):
        asc = _fold(raw[t], w[t], np.argsort(ids[t], kind="stable"))
        assert np.array_equal(got[t], asc), t
        rank_differs += int(not np.array_equal(asc, _fold(raw[t], w[t], range(8))))
    assert rank_differs > 0
