"""The third named caller, speccheck/moe_ref.py:499 moe_block(x, w: BlockWeights, g, form="ref"),
on the device: dense Hugging Face bf16 weights (gate_up [256, 1024, 2048], down [256, 2048, 512],
the shared expert) read in place by the gather-GEMV decode kernels.

The layer is the seeded synthetic layer (seed 0, layer 0) in the dense layout: its Q4_K matrices
dequantised to bf16. tests/golden/moe_ref_t4.npz holds the reference's own moe_ref.moe_block
outputs on 4 tokens for the same tensors, in its "ref" form (bf16 accumulate) and its "exact" form
(f64). Bars (written here):
* routing: the same 8 experts per token as the reference, in the same rank order except among
  experts whose bf16 logits tie exactly (torch.topk leaves their order unspecified; the library
  puts the lower index first); router logits within one bf16 ulp (the F.linear order of the
  reference is oneDNN's, the library's is its declared one). Per-slot stages are compared slot by
  slot after matching the slots by expert id;
* every "ref"-form stage tensor (bf16) against the reference's: at least 99 % of the elements
  bit-identical, and the rel-L2 distance below 2e-3 (one bf16 ulp is 2^-8 relative at most: the
  two sides round the same f32 sums, whose order differs, at the same points);
* the block output at least as close to the exact f64 form as the reference's own "ref" output
  is (rel-L2 within 1.25x of the reference's, plus 1e-6);
* the same layer through b200moe.moe.moe_block (f32 throughout) against the f64 oracle on the
  dense weights with the same routing: rel-L2 < 1e-5, the decode path's bar;
* forms other than [REF], injection knobs and wrong dtypes are refused with a tag.
"""
import numpy as np
import pytest

from conftest import golden, host_layer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dense0(cuda):
    from b200moe.engine import DeviceLayer
    return DeviceLayer.synthetic_dense(0, 0, cuda)


@pytest.fixture(scope="module")
def weights(dense0):
    import torch
    from b200moe import moe_ref
    from b200moe.geometry import E, H, I
    L = dense0
    t = {"router": L.router_w.reshape(E, H), "gate_up": L.gate.view(torch.bfloat16).reshape(E, 2 * I, H),
         "down": L.down.view(torch.bfloat16).reshape(E, H, I),
         "shared_gate": L.sh_gate.view(torch.bfloat16).reshape(I, H),
         "shared_up": L.sh_up.view(torch.bfloat16).reshape(I, H),
         "shared_down": L.sh_down.view(torch.bfloat16).reshape(H, I),
         "shared_scalar_gate": L.sh_gate_w.reshape(1, H)}
    w = moe_ref.BlockWeights("layer0", t)
    w.shapes_ok(moe_ref.Geometry())
    return w


def _bits(t):
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _bf(bits):
    from oracle.bf16 import bf16_bits_to_f32
    return bf16_bits_to_f32(bits).astype(np.float64)


def test_moe_ref_ref_form_against_reference(cuda, weights):
    import torch
    from b200moe import moe_ref
    G = golden("moe_ref_t4.npz")
    x = torch.from_numpy(G["x_bits"].view(np.int16)).view(torch.bfloat16).to(cuda)
    st = moe_ref.moe_block(x, weights, moe_ref.Geometry(), "ref")
    torch.cuda.synchronize()
    assert st["form"] == moe_ref.Form()
    ids, rids = st["topk_ids"].cpu().numpy(), G["ref_topk_ids"]
    logit_bits = _bits(st["router_logits"])
    perm = np.zeros_like(ids)  # perm[t, k]: our slot holding the reference's slot-k expert
    for t in range(ids.shape[0]):
        assert sorted(ids[t]) == sorted(rids[t]), t
        for k in range(ids.shape[1]):
            j = int(np.nonzero(ids[t] == rids[t, k])[0][0])
            perm[t, k] = j
            if j != k:  # a rank-order difference is allowed only between exactly tied logits
                assert logit_bits[t, rids[t, k]] == logit_bits[t, ids[t, k]], (t, k)
    dl = np.abs(logit_bits.astype(np.int32) - G["ref_router_logits"].astype(np.int32))
    assert dl.max() <= 1 and (dl > 0).mean() <= 0.01
    report = {}
    for k in ("topk_weights", "expert_raw", "routed_sum", "shared_raw", "shared_gate_prob", "shared_out",
              "combined_out"):
        got, want = _bits(st[k]), G["ref_" + k]
        if k in ("topk_weights", "expert_raw"):  # slot-indexed: the reference's slot order
            got = np.stack([got[t][perm[t]] for t in range(got.shape[0])])
        assert got.shape == want.shape, k
        same = float((got == want).mean())
        a, b = _bf(got), _bf(want)
        rel = float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))
        report[k] = (same, rel)
        assert same >= 0.99 and rel < 2e-3, (k, same, rel)
    exact = G["exact_combined_out"]
    ours = float(np.linalg.norm(_bf(_bits(st["combined_out"])) - exact) / np.linalg.norm(exact))
    theirs = float(np.linalg.norm(_bf(G["ref_combined_out"]) - exact) / np.linalg.norm(exact))
    print("moe_ref ref form: identical fraction / rel-L2 per stage %s; distance to exact: ours %.3e, "
          "reference %.3e" % ({k: ("%.4f" % v[0], "%.1e" % v[1]) for k, v in report.items()}, ours, theirs))
    assert ours <= 1.25 * theirs + 1e-6


def test_dense_layer_f32_path_against_oracle(cuda, dense0):
    """The dense layer through the f32 decode path (b200moe.moe.moe_block) vs the f64 restatement
    of engine/m3_forward.py:430-476 on the same bf16 weights and the same routing."""
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    host = host_layer(0, 0, bf16_weights=True)
    for T, stream in ((1, 30), (5, 31), (16, 32)):
        xb = synth.tokens(0, T, stream=stream)
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
        out, info = moe.moe_block(x, dense0, 0, check=True)
        torch.cuda.synchronize()
        xf = bf16_bits_to_f32(xb)
        r = OM.router(xf, host.wg)
        ids = info["ids"].cpu().numpy()
        assert (ids == r["ids"]).all(), T
        want = OM.moe_block_f64(xf, host, r["ids"], r["w_bf16"])["out"]
        c = OM.compare(out.cpu().numpy(), want)
        assert c["rel_l2"] < 1e-5, (T, c)


def test_moe_ref_refusals(cuda, weights):
    import torch
    from b200moe import moe_ref
    from b200moe.moe import Refused
    x = torch.zeros((2, 2048), dtype=torch.bfloat16, device=cuda)
    for form in ("exact", "spec", "cast_after", "rank_order"):
        with pytest.raises(Refused) as ei:
            moe_ref.moe_block(x, weights, form=form)
        assert ei.value.tag == "form"
    with pytest.raises(Refused) as ei:
        moe_ref.moe_block(x, weights, swap_halves=True)
    assert ei.value.tag == "injection"
    with pytest.raises(Refused) as ei:
        moe_ref.moe_block(x.float(), weights)
    assert ei.value.tag == "dtype"
    with pytest.raises(Refused) as ei:
        moe_ref.moe_block(x.reshape(2, 1, 2048), weights)
    assert ei.value.tag == "batch"
    with pytest.raises(Refused):
        moe_ref.Form.named("nonsense")
