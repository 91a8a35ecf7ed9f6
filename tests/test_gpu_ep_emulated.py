"""The expert-parallel data plane on one GPU: every rank's stages run in turn on cuda:0 and the
two all-to-all exchanges are done by permuting the row blocks between the ranks' buffers.

This checks the device kernels of b200moe_ep_pack / b200moe_ep_experts / b200moe_ep_combine
through the C ABI exactly as the NCCL ranks use them (test_gpu_ep.py runs them over NCCL when
the box has several GPUs):
* the pack's rows and positions equal a host restatement of the dispatch rule (every token once
  per destination that owns one of its experts, ascending token order; all own tokens to the own
  block; empty rows with ids -1);
* the combined outputs equal the single-GPU prefill of all tokens within rel-L2 1e-5 (only the
  association of the routed sum differs), with identical routing ids, for W = 2, 4, 8.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROW = 4160


@pytest.fixture(scope="module")
def layer3(cuda):
    from b200moe.engine import DeviceLayer
    return DeviceLayer.synthetic(3, 0, cuda)


def _host_pack(ids, rank, world):
    """Expected pos [T, W] and row ids per destination block."""
    T = ids.shape[0]
    per = 256 // world
    pos = np.full((T, world), -1, np.int32)
    for d in range(world):
        own = (ids >= d * per) & (ids < (d + 1) * per)
        take = np.ones(T, bool) if d == rank else own.any(axis=1)
        pos[take, d] = np.arange(int(take.sum()))
    return pos


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_stages_emulated_match_single_gpu(cuda, layer3, world):
    import torch
    from b200moe import _abi, moe, synth
    from b200moe.geometry import RMS_EPS
    T_all = 512
    T = T_all // world
    xb = synth.tokens(3, T_all, stream=9)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    ref, info = moe.moe_block(x, layer3, path="prefill")
    ws = torch.empty(_abi.prefill_workspace_size(T_all), dtype=torch.uint8, device=cuda)
    routed, sends, poss = [], [], []
    for r in range(world):
        x16 = torch.empty((T, 2048), dtype=torch.float16, device=cuda)
        ids = torch.empty((T, 8), dtype=torch.int32, device=cuda)
        wb = torch.empty((T, 8), dtype=torch.int16, device=cuda)
        sg = torch.empty((T,), dtype=torch.float32, device=cuda)
        _abi.moe_route(x[r * T:(r + 1) * T], _abi.BF16, None, RMS_EPS, T, layer3.abi(), x16, ids, wb, sg, ws)
        send = torch.zeros((world, T, ROW), dtype=torch.uint8, device=cuda)
        pos = torch.empty((T, world), dtype=torch.int32, device=cuda)
        _abi.ep_pack(x16, ids, wb, T, r, world, send, pos)
        torch.cuda.synchronize()
        # the pack against its host restatement
        idn = ids.cpu().numpy()
        want = _host_pack(idn, r, world)
        assert np.array_equal(pos.cpu().numpy(), want), r
        sv = send.cpu().numpy()
        x16n = x16.cpu().numpy().view(np.uint8).reshape(T, 4096)
        for d in range(world):
            for t in np.nonzero(want[:, d] >= 0)[0]:
                p = want[t, d]
                assert np.array_equal(sv[d, p, :4096], x16n[t])
                assert np.array_equal(sv[d, p, 4096:4128].view(np.int32), idn[t])
            n = int((want[:, d] >= 0).sum())
            assert (sv[d, n:, 4096:4128].view(np.int32) == -1).all()
        routed.append((ids, sg))
        sends.append(send)
        poss.append(pos)
    partials = []
    for d in range(world):  # rank d receives block d of every source
        recv = torch.stack([sends[s][d] for s in range(world)]).contiguous()
        partial = torch.empty((world, T, 2048), dtype=torch.float32, device=cuda)
        _abi.ep_experts(recv, T, d, world, routed[d][1], layer3.abi(), partial, ws)
        assert _abi.prefill_status(ws, world * T) == 0
        partials.append(partial)
    outs = []
    for s in range(world):  # rank s gets block s of every rank's partials back
        ret = torch.stack([partials[d][s] for d in range(world)]).contiguous()
        out = torch.full((T, 2048), float("nan"), dtype=torch.float32, device=cuda)
        _abi.ep_combine(ret, poss[s], T, world, out, False)
        outs.append(out)
    torch.cuda.synchronize()
    o = torch.cat(outs)
    assert torch.equal(torch.cat([r[0] for r in routed]), info["ids"])
    rel = float(torch.linalg.norm(o - ref) / torch.linalg.norm(ref))
    assert rel < 1e-5, rel
    # accumulate mode adds onto what is there
    acc = torch.ones((T, 2048), dtype=torch.float32, device=cuda)
    ret = torch.stack([partials[d][0] for d in range(world)]).contiguous()
    _abi.ep_combine(ret, poss[0], T, world, acc, True)
    torch.cuda.synchronize()
    assert torch.allclose(acc, outs[0] + 1.0, rtol=1e-6, atol=1e-3)
