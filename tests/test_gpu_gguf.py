"""A layer read from a GGUF file (qwen3.6-35b-a3b_b200/gguf.py) runs the MoE block with the same
bits as the same layer built in memory: the seeded synthetic layer is written out as a GGUF v3
file (Q4_K expert and shared tensors, bf16 router and gate), read back through
gguf.device_engine, and both go through moe_block on the decode and prefill paths."""
import numpy as np
import pytest

from test_gguf_loader import BF16, Q4K, E, H, I, write_gguf

pytestmark = pytest.mark.gpu


def test_gguf_layer_equals_in_memory_layer(cuda, tmp_path):
    import torch
    from b200moe import gguf, moe, synth
    from b200moe.engine import DeviceLayer
    L = DeviceLayer.synthetic(5, 7, cuda)
    host = lambda t: t.reshape(-1).view(torch.uint8).cpu().numpy().tobytes()  # noqa: E731
    p = "blk.7."
    tensors = [(p + "ffn_gate_exps.weight", (H, I, E), Q4K, {0: host(L.gate)}),
               (p + "ffn_up_exps.weight", (H, I, E), Q4K, {0: host(L.up)}),
               (p + "ffn_down_exps.weight", (I, H, E), Q4K, {0: host(L.down)}),
               (p + "ffn_gate_shexp.weight", (H, I), Q4K, {0: host(L.sh_gate)}),
               (p + "ffn_up_shexp.weight", (H, I), Q4K, {0: host(L.sh_up)}),
               (p + "ffn_down_shexp.weight", (I, H), Q4K, {0: host(L.sh_down)}),
               (p + "ffn_gate_inp.weight", (H, E), BF16, {0: host(L.router_w)}),
               (p + "ffn_gate_inp_shexp.weight", (H, 1), BF16, {0: host(L.sh_gate_w)})]
    path = str(tmp_path / "layer7.gguf")
    write_gguf(path, tensors)
    del tensors
    G = gguf.device_engine(path, device=cuda)
    assert len(G.layers) == 1
    xb = synth.tokens(5, 40, stream=9)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    for path_ in ("decode", "prefill"):
        a, ia = moe.moe_block(x, L, 0, path=path_)
        b, ib = moe.moe_block(x, G.layers[0], 0, path=path_)
        torch.cuda.synchronize()
        assert torch.equal(ia["ids"], ib["ids"]) and torch.equal(a, b), path_


def test_gguf_published_layout_equals_in_memory_layer(cuda, tmp_path):
    """The published Q4_K_M file's layer layout -- Q4_K gate / up, Q5_K down, Q8_0 shared expert,
    F32 router and shared gate, F32 post-attention norm weight -- written as a GGUF file and read
    back (types from the file) gives the same bits as the layer built in memory: one token (the
    persistent kernel's format variant), several (the gather-GEMV kernels), and the residual
    stack (norm weight applied)."""
    import torch
    from oracle import kquants
    from test_gguf_loader import F32, Q5K, Q80
    from b200moe import gguf, moe, synth
    from b200moe.engine import DeviceEngine, DeviceLayer
    base = DeviceLayer.synthetic(5, 8, cuda)
    down = kquants.random_blocks("Q5_K", E * H * I // 256, 81).reshape(-1)
    sh = {k: kquants.random_blocks("Q8_0", n // 32, s).reshape(-1)
          for k, n, s in (("sh_gate", I * H, 82), ("sh_up", I * H, 83), ("sh_down", H * I, 84))}
    router = base.router_w.float().cpu().numpy()
    shgate = base.sh_gate_w.float().cpu().numpy()
    nw = (1.0 + np.random.default_rng(85).normal(0, 0.05, H)).astype(np.float32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    L = DeviceLayer(base.gate, base.up, dev(down), dev(sh["sh_gate"]), dev(sh["sh_up"]), dev(sh["sh_down"]),
                    dev(router), dev(shgate), norm_w=dev(nw), down_type="Q5_K", sh_type="Q8_0")
    host = lambda t: t.reshape(-1).view(torch.uint8).cpu().numpy().tobytes()  # noqa: E731
    p = "blk.8."
    tensors = [(p + "ffn_gate_exps.weight", (H, I, E), Q4K, {0: host(base.gate)}),
               (p + "ffn_up_exps.weight", (H, I, E), Q4K, {0: host(base.up)}),
               (p + "ffn_down_exps.weight", (I, H, E), Q5K, {0: down.tobytes()}),
               (p + "ffn_gate_shexp.weight", (H, I), Q80, {0: sh["sh_gate"].tobytes()}),
               (p + "ffn_up_shexp.weight", (H, I), Q80, {0: sh["sh_up"].tobytes()}),
               (p + "ffn_down_shexp.weight", (I, H), Q80, {0: sh["sh_down"].tobytes()}),
               (p + "ffn_gate_inp.weight", (H, E), F32, {0: router.tobytes()}),
               (p + "ffn_gate_inp_shexp.weight", (H,), F32, {0: shgate.tobytes()}),
               (p + "post_attention_norm.weight", (H,), F32, {0: nw.tobytes()})]
    path = str(tmp_path / "layer8.gguf")
    write_gguf(path, tensors)
    del tensors
    G = gguf.device_engine(path, device=cuda)
    F = G.layers[0]
    assert (F.down_type, F.sh_type, F.router_w.dtype) == ("Q5_K", "Q8_0", torch.float32)
    xb = synth.tokens(5, 3, stream=10)
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    for T in (1, 3):
        a, ia = moe.moe_block(x[:T], L)
        b, ib = moe.moe_block(x[:T], F)
        torch.cuda.synchronize()
        assert torch.equal(ia["ids"], ib["ids"]) and torch.equal(a, b), T
    r0 = x[:1].float()
    ra, rb = r0.clone(), r0.clone()
    moe.moe_stack(ra, DeviceEngine([L]))
    moe.moe_stack(rb, G)
    torch.cuda.synchronize()
    assert torch.isfinite(ra).all() and torch.equal(ra, rb)
