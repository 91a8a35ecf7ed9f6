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
