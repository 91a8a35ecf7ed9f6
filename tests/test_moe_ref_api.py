"""b200moe.moe_ref -- the reference-shaped API of speccheck/moe_ref.py (Geometry, Form,
BlockWeights, moe_block) -- on CPU: the types carry the reference's fields and arms, and every
refusal (a non-[REF] form, an injection knob, a wrong dtype, shape or batch) happens before any
device work."""
import pytest
import torch


def test_geometry_and_form_fields():
    from b200moe import moe_ref
    g = moe_ref.Geometry()
    assert (g.hidden_size, g.num_experts, g.top_k, g.moe_intermediate_size, g.two_i) == (2048, 256, 8, 512, 1024)
    assert g.expert_bytes == (1024 * 2048 + 2048 * 512) * 2 and g.n_blocks == 41
    ref = moe_ref.Form.named("ref")
    assert ref == moe_ref.Form() and ref.accumulate == "bf16" and ref.weight_cast == "before"
    assert moe_ref.Form.named("exact").router_dtype == "f64"
    assert moe_ref.Form.named("rank_order").order == "rank"


def test_block_weights_shapes_ok():
    from b200moe import moe_ref
    from b200moe.moe import Refused
    g = moe_ref.Geometry()
    shapes = moe_ref._shapes(g)
    t = {k: torch.empty(0, dtype=torch.bfloat16).new_empty(v) for k, v in shapes.items() if k != "gate_up"}
    w = moe_ref.BlockWeights("layer0", t)
    w.shapes_ok(g, roles=tuple(k for k in shapes if k != "gate_up"))
    with pytest.raises(Refused) as ei:
        w.shapes_ok(g)
    assert ei.value.tag == "shape"
    t["gate_up"] = torch.empty(shapes["gate_up"], dtype=torch.float32)
    with pytest.raises(Refused) as ei:
        moe_ref.BlockWeights("layer0", t).shapes_ok(g)
    assert ei.value.tag == "dtype"


@pytest.mark.parametrize("kw,tag", [(dict(form="exact"), "form"), (dict(form="accum_f32"), "form"),
                                    (dict(expert_index_shift=1), "injection"), (dict(transpose_stack=True), "injection")])
def test_refusals_before_device_work(kw, tag):
    from b200moe import moe_ref
    from b200moe.moe import Refused
    w = moe_ref.BlockWeights("layer0", {})          # never touched: the call is refused first
    with pytest.raises(Refused) as ei:
        moe_ref.moe_block(torch.zeros((1, 2048), dtype=torch.bfloat16), w, **kw)
    assert ei.value.tag == tag


def test_refuses_input_forms():
    from b200moe import moe_ref
    from b200moe.moe import Refused
    w = moe_ref.BlockWeights("layer0", {})
    for x, tag in ((torch.zeros((1, 2048)), "dtype"), (torch.zeros((2, 1, 2048), dtype=torch.bfloat16), "batch"),
                   (torch.zeros((1, 1024), dtype=torch.bfloat16), "shape")):
        with pytest.raises(Refused) as ei:
            moe_ref.moe_block(x, w)
        assert ei.value.tag == tag
