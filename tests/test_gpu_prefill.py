"""The prefill path (token sort + tcgen05 grouped GEMMs, b200moe_moe_prefill) vs the oracle.

Parity bar (written here): routing ids bit-exact against the declared-order C restatement
(the same router as decode); block output against the f64 restatement of
engine/m3_forward.py:430-476 with the same ids within rel-L2 1e-3 and
max-abs / max|ref| 2e-3. The tensor cores take fp16 operands (weights dequantised from Q4_K
to fp16, activations rounded to fp16), so the f32-level agreement of the decode path is not
expected here; the bar above is.
"""
import numpy as np
import pytest

from conftest import host_layer

pytestmark = pytest.mark.gpu
REL_L2, MAX_ABS_NORM = 1e-3, 2e-3


@pytest.fixture(scope="module")
def layer3(cuda):
    from b200moe.engine import DeviceLayer
    return DeviceLayer.synthetic(3, 0, cuda)


def _run(cuda, L, xb):
    import torch
    from b200moe import moe
    T = xb.shape[0]
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    out, info = moe.moe_block(x, L, 0, path="prefill")
    torch.cuda.synchronize()
    assert moe.prefill_status(T, cuda) == 0
    return out.cpu().numpy(), info["ids"].cpu().numpy()


def _check(xb, out, ids, Lh, sample=None):
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    x = bf16_bits_to_f32(xb)
    r = OM.router(x, Lh.wg, Lh.bias)
    assert (ids == r["ids"]).all()
    rows = np.arange(x.shape[0]) if sample is None else sample
    ref = OM.moe_block_f64(x[rows], Lh, ids[rows], r["w_bf16"][rows])["out"]
    c = OM.compare(out[rows], ref)
    assert c["rel_l2"] < REL_L2 and c["max_abs_norm"] < MAX_ABS_NORM, c
    return c


@pytest.mark.parametrize("T", [1, 17, 256])
def test_prefill_vs_oracle(cuda, layer3, T):
    from b200moe import synth
    xb = synth.tokens(3, T, stream=0)
    out, ids = _run(cuda, layer3, xb)
    _check(xb, out, ids, host_layer(3, 0))


def test_prefill_config3_4096(cuda, layer3):
    """Config 3 size (4096 tokens; the shared expert spans 22 tiles of at most 192 tokens): ids and
    outputs for every token against the f64 oracle (the achieved margin is printed),
    deterministic across runs."""
    from b200moe import synth
    xb = synth.tokens(3, 4096, stream=1)
    out, ids = _run(cuda, layer3, xb)
    out2, ids2 = _run(cuda, layer3, xb)
    assert (ids == ids2).all() and np.array_equal(out, out2)
    c = _check(xb, out, ids, host_layer(3, 0))
    print("config-3 prefill, all 4096 tokens: rel_l2 %.3e (bar %.0e), max_abs_norm %.3e (bar %.0e)"
          % (c["rel_l2"], REL_L2, c["max_abs_norm"], MAX_ABS_NORM))
    assert np.isfinite(out).all()


def test_prefill_repeat_bit_identical_8192(cuda, layer3):
    """8192 tokens: each GEMM CTA walks dozens of tiles, so every ring, TMEM stage and epilogue
    staging buffer wraps many times; a buffer reused before its last reader finished would show
    up as bits that change between runs. Three runs give identical bits."""
    from b200moe import synth
    xb = synth.tokens(3, 8192, stream=4)
    out, ids = _run(cuda, layer3, xb)
    for _ in range(2):
        out2, ids2 = _run(cuda, layer3, xb)
        assert (ids == ids2).all() and np.array_equal(out, out2)
    assert np.isfinite(out).all()


def test_prefill_matches_decode_routing_and_output(cuda, layer3):
    import torch
    from b200moe import moe, synth
    xb = synth.tokens(3, 96, stream=2)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    a, ia = moe.moe_block(x, layer3, path="prefill")
    b, ib = moe.moe_block(x, layer3, path="decode")
    torch.cuda.synchronize()
    assert torch.equal(ia["ids"], ib["ids"])
    rel = float(torch.linalg.norm(a - b) / torch.linalg.norm(b))
    assert rel < REL_L2


def test_prefill_zipf_skew(cuda):
    """Config 2 law at 512 tokens: skewed expert load (several experts above 192 tokens,
    i.e. multi-chunk groups), many experts idle."""
    from b200moe import synth
    from b200moe.engine import DeviceLayer
    L = DeviceLayer.synthetic(2, 0, cuda, bias=True)
    xb = synth.tokens(2, 512, stream=3)
    out, ids = _run(cuda, L, xb)
    counts = np.bincount(ids.reshape(-1), minlength=256)
    assert counts.max() > 256 and (counts == 0).any()
    sample = np.sort(np.random.default_rng(1).choice(512, 32, replace=False))
    _check(xb, out, ids, host_layer(2, 0, bias=True), sample)
    del L


def test_stack_prefill_teacher_forced(cuda):
    """Two layers of the config-4 stack on the prefill path (resid += moe(rmsnorm(resid)))."""
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    from b200moe.engine import DeviceEngine
    eng = DeviceEngine.synthetic(4, 2, cuda)
    T = 80
    resid = torch.from_numpy(bf16_bits_to_f32(synth.tokens(4, T, stream=11)).copy()).to(cuda)
    for l in range(2):
        before = resid.cpu().numpy().copy()
        ids = torch.empty((1, T, 8), dtype=torch.int32, device=cuda)
        moe.moe_stack_prefill(resid, DeviceEngine([eng.layers[l]]), ids_out=ids)
        torch.cuda.synchronize()
        assert moe.prefill_status(T, cuda) == 0
        Lh = host_layer(4, l)
        xn = OM.rmsnorm(before)
        r = OM.router(xn, Lh.wg)
        assert (ids.cpu().numpy().reshape(T, 8) == r["ids"]).all(), l
        sample = np.arange(0, T, 5)
        ref = before[sample].astype(np.float64) + OM.moe_block_f64(xn[sample], Lh, r["ids"][sample],
                                                                   r["w_bf16"][sample])["out"]
        c = OM.compare(resid.cpu().numpy()[sample], ref)
        assert c["rel_l2"] < REL_L2, (l, c)
    del eng


@pytest.mark.parametrize("W", [2, 4])
def test_expert_ranges_as_in_expert_parallelism(cuda, layer3, W):
    """The expert-parallel decomposition on one GPU, through the same C-ABI calls the NCCL path
    makes: route all tokens once; for each rank r, one b200moe_moe_experts call over all tokens
    with its expert range [256r/W, 256(r+1)/W) and the shared expert on its own rows only; the
    sum of the W partial rows in ascending rank order must equal the single-call prefill
    (rel-L2 1e-5: only the association of the routed sum differs)."""
    import torch
    from b200moe import _abi, moe, synth
    from b200moe.ep import device_route_fn
    T = 512
    xb = synth.tokens(3, T, stream=5)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    ref, info = moe.moe_block(x, layer3, 0, path="prefill")
    ws = lambda n: moe.prefill_workspace(n, cuda)
    x16, ids, wb, sg = device_route_fn(layer3, ws)(x)
    Tr = T // W
    out = None
    for r in range(W):
        part = torch.empty((T, 2048), dtype=torch.float32, device=cuda)
        _abi.moe_experts(x16, T, ids, wb, 256 * r // W, 256 * (r + 1) // W, sg[r * Tr:(r + 1) * Tr], layer3.abi(),
                         part, False, ws(T), sh_rows=(r * Tr, (r + 1) * Tr))
        out = part if out is None else out + part
    torch.cuda.synchronize()
    assert moe.prefill_status(T, cuda) == 0
    assert torch.equal(ids, info["ids"].reshape(T, 8))
    rel = float(torch.linalg.norm(out - ref.reshape(T, 2048)) / torch.linalg.norm(ref))
    assert torch.isfinite(out).all() and rel < 1e-5, rel


def test_block_stages_match_oracle_stages(cuda, layer3):
    """moe_block_stages (engine/block_forward.py:670's stage dictionary) against the f64
    restatement's stage tensors on the same ids: router stages bit-exact, every numeric stage
    within the prefill bar, combined_out bit-identical to the prefill block output."""
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    T = 5
    xb = synth.tokens(3, T, stream=6)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    st = moe.moe_block_stages(x, layer3, 0)
    blk, _ = moe.moe_block(x, layer3, 0, path="prefill")
    torch.cuda.synchronize()
    assert moe.prefill_status(T, cuda) == 0
    for k in ("shared_raw", "shared_gate_prob", "shared_out", "router_logits", "topk_ids", "topk_weights",
              "topk_weights_f32", "expert_raw", "routed_sum", "combined_out"):
        assert k in st, k
    assert st["expert_raw"].shape == (T, 8, 2048) and st["shared_gate_prob"].shape == (T, 1)
    assert torch.equal(st["combined_out"], blk.reshape(T, 2048))
    Lh = host_layer(3, 0)
    xf = bf16_bits_to_f32(xb)
    r = OM.router(xf, Lh.wg, Lh.bias)
    ids = st["topk_ids"].cpu().numpy()
    assert (ids == r["ids"]).all()
    assert (st["topk_weights"].view(torch.int16).cpu().numpy().view(np.uint16) == r["w_bf16"]).all()
    ref = OM.moe_block_f64(xf, Lh, ids, r["w_bf16"])
    pairs = (("shared_raw", "shared_raw"), ("shared_out", "shared_out"), ("routed_sum", "routed"),
             ("combined_out", "out"))
    for mine, theirs in pairs:
        c = OM.compare(st[mine].cpu().numpy(), ref[theirs])
        assert c["rel_l2"] < REL_L2 and c["max_abs_norm"] < MAX_ABS_NORM, (mine, c)
    for k in range(8):
        c = OM.compare(st["expert_raw"][:, k].cpu().numpy(), ref["expert_raw"][:, k])
        assert c["rel_l2"] < REL_L2 and c["max_abs_norm"] < MAX_ABS_NORM, ("expert_raw", k, c)
    g = st["shared_gate_prob"].reshape(T).cpu().numpy().astype(np.float64)
    assert np.max(np.abs(g - ref["shared_gate_prob"])) < 1e-6


@pytest.mark.parametrize("T", [17, 300, 1024, 2368, 4096])
def test_route_stage_every_router_tile(cuda, layer3, T):
    """The prefill router: up to 576 tokens take the row kernel (a warp per four router rows, a lane
    per K chunk), more the tiled GEMM, whose token tile (8 .. 64 tokens per CTA) is picked by
    batch size so the busiest SM has the fewest rows: on 148 SMs 17 and 300 tokens take the row
    kernel, 1024 the 32-token tile, 2368 the 64-token one and 4096 the 56-token one. Each output
    is the same declared sequence of operations, so ids and R5 weights are bit-exact against the
    C restatement on every path."""
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import _abi, synth
    from b200moe.geometry import RMS_EPS
    xb = synth.tokens(3, T, stream=12)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    x16 = torch.empty((T, 2048), dtype=torch.float16, device=cuda)
    ids = torch.empty((T, 8), dtype=torch.int32, device=cuda)
    wb = torch.empty((T, 8), dtype=torch.int16, device=cuda)
    sg = torch.empty((T,), dtype=torch.float32, device=cuda)
    ws = torch.empty(_abi.prefill_workspace_size(T), dtype=torch.uint8, device=cuda)
    _abi.moe_route(x, _abi.BF16, None, RMS_EPS, T, layer3.abi(), x16, ids, wb, sg, ws)
    torch.cuda.synchronize()
    r = OM.router(bf16_bits_to_f32(xb), host_layer(3, 0).wg)
    assert (ids.cpu().numpy() == r["ids"]).all()
    assert (wb.cpu().numpy().view(np.uint16) == r["w_bf16"]).all()
