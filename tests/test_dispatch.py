"""The block API's path choice (qwen3.6-35b-a3b_b200/moe.py), on CPU with the library's entry
points replaced by recorders: Q4_K layers take the grouped GEMMs from PREFILL_MIN_TOKENS tokens
on and the decode kernels below; layers in the published file's other block formats stay on the
decode kernels at every token count; path="prefill" refuses them before any launch; the
prefill-path stack runs them through b200moe_stack_decode on the caller's workspace."""
import pytest


@pytest.fixture
def rec(monkeypatch):
    import torch
    from b200moe import _abi, moe
    calls = []
    monkeypatch.setattr(_abi, "moe_prefill", lambda *a, **k: calls.append(("prefill", a[4])))
    monkeypatch.setattr(_abi, "moe_decode", lambda *a, **k: calls.append(("decode", a[2])))
    monkeypatch.setattr(_abi, "stack_decode", lambda r, T, layers, eps, ids, ws, stream=None:
                        calls.append(("stack_decode", T, len(layers), ws.numel())))
    monkeypatch.setattr(_abi, "decode_workspace_size", lambda T: 1000 * T)
    monkeypatch.setattr(moe, "workspace", lambda T, dev: torch.empty(1000 * T, dtype=torch.uint8))
    monkeypatch.setattr(moe, "prefill_workspace", lambda T, dev: torch.empty(5000 * T, dtype=torch.uint8))
    return calls


def _layer(down="Q4_K", sh="Q4_K"):
    from test_bench_accounting import _layer as mk  # a layer of uninitialised CPU tensors
    return mk(down, sh)


@pytest.mark.parametrize("T,want", [(1, "decode"), (4, "decode"), (12, "decode"), (13, "prefill"), (64, "prefill")])
def test_q4k_layer_auto_path(rec, T, want):
    import torch
    from b200moe import moe
    moe.moe_block(torch.zeros((T, 2048)), _layer())
    assert rec == [(want, T)]


@pytest.mark.parametrize("T", [1, 10, 512])
def test_published_format_layer_stays_on_decode(rec, T):
    import torch
    from b200moe import moe
    moe.moe_block(torch.zeros((T, 2048)), _layer("Q5_K", "Q8_0"))
    assert rec == [("decode", T)]


def test_prefill_path_refuses_published_format_layer(rec):
    import torch
    from b200moe import moe
    with pytest.raises(moe.Refused) as ei:
        moe.moe_block(torch.zeros((16, 2048)), _layer("Q6_K", "Q4_K"), path="prefill")
    assert ei.value.tag == "format" and rec == []


def test_prefill_stack_mixes_paths_per_layer(rec):
    import torch
    from b200moe import moe
    from b200moe.engine import DeviceEngine
    eng = DeviceEngine([_layer(), _layer("Q5_K", "Q8_0"), _layer()])
    resid = torch.zeros((32, 2048), dtype=torch.float32)
    moe.moe_stack_prefill(resid, eng)
    # the Q4_K layers on the grouped GEMMs; the other on the decode kernels, reusing the
    # (larger) prefill workspace instead of allocating
    assert rec == [("prefill", 32), ("stack_decode", 32, 1, 5000 * 32), ("prefill", 32)]


def test_refusals_before_any_call(rec):
    import torch
    from b200moe import moe
    L = _layer()
    with pytest.raises(moe.Refused):
        moe.moe_block(torch.zeros((2, 1024)), L)
    with pytest.raises(moe.Refused):
        moe.moe_block(torch.zeros((2, 2048), dtype=torch.float64), L)
    with pytest.raises(moe.Refused):
        moe.moe_block(torch.zeros((2, 2048)), L, path="gemm")
    with pytest.raises(moe.Refused):
        moe.moe_block(torch.zeros((2, 2048)), L, probe_row=0)
    assert rec == []


def test_no_tokens_give_empty_results_without_device_work(rec):
    """As the reference's loop does for B*T = 0: empty outputs in the input's leading shape."""
    import torch
    from b200moe import moe
    from b200moe.engine import DeviceEngine
    L = _layer()
    out, info = moe.moe_block(torch.zeros((1, 0, 2048)), L)
    assert tuple(out.shape) == (1, 0, 2048) and tuple(info["ids"].shape) == (1, 0, 8) and info["used"] == 0
    r = moe.moe_router(torch.zeros((0, 2048)), L)
    assert tuple(r["router_logits"].shape) == (0, 256) and tuple(r["topk_ids"].shape) == (0, 8)
    resid = torch.zeros((0, 2048), dtype=torch.float32)
    assert moe.moe_stack(resid, DeviceEngine([L])) is resid
    assert moe.moe_stack_prefill(resid, DeviceEngine([L])) is resid
    st = moe.moe_block_stages(torch.zeros((0, 2048)), L)
    assert tuple(st["expert_raw"].shape) == (0, 8, 2048) and tuple(st["combined_out"].shape) == (0, 2048)
    assert rec == []
