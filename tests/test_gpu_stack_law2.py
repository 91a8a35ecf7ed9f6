"""The config-4 stack under a second, well-conditioned weight law.

Under the BASELINE field law every Q4_K weight has a mean of about +1.2, so after one layer the
residual is dominated by one common direction: every token's RMSNorm input is nearly the same and
routing collapses onto the same experts (the first-law stack tests still check every layer's
arithmetic, but on near-identical inputs past layer 1). The second law keeps the same seeded
blocks and scales each super-block's f16 d by 2^-6 and dmin by 2^-2, which centres the weights
(E[w] ~ 0): the residual stays O(1), tokens stay distinct and routing stays diverse.

Per layer, teacher-forced as tests/test_gpu_stack.py: the oracle takes the device's residual
entering the layer; ids bit-exact against the declared-order router, the residual after the layer
within rel-L2 1e-5 of the f64 block. The stack is also checked to be non-degenerate (distinct
experts per layer, token similarity, residual size), and the counts are printed. Token counts
1 (persistent kernel) and 4, 12 (grouped decode kernels).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
N_LAYERS = 4


def host_layer2(seed, layer):
    from oracle import q4k
    from oracle.moe import HostLayer
    from b200moe import synth
    from b200moe.geometry import KIND_OF, stream_id

    def blocks(kind, first, n):
        return synth.law2_blocks(q4k.synth_blocks(seed, stream_id(layer, KIND_OF[kind]), first, n))

    return HostLayer(blocks, synth.router_w(seed, layer), synth.shared_gate_w(seed, layer))


@pytest.fixture(scope="module")
def engine_law2(cuda):
    from b200moe import synth
    from b200moe.engine import DeviceEngine, DeviceLayer
    layers = []
    for l in range(N_LAYERS):
        L = DeviceLayer.synthetic(4, l, cuda)
        for t in (L.gate, L.up, L.down, L.sh_gate, L.sh_up, L.sh_down):
            synth.law2_blocks_(t)
        layers.append(L)
    return DeviceEngine(layers)


def test_law2_bytes_match_host(cuda, engine_law2):
    """Sampled blocks of every kind: the device scaling equals the host mirror byte for byte."""
    from oracle import q4k
    from b200moe import synth
    from b200moe.geometry import KIND_OF, stream_id
    L = engine_law2.layers[1]
    rng = np.random.default_rng(0)
    for kind, t in (("gate", L.gate), ("up", L.up), ("down", L.down), ("sh_gate", L.sh_gate),
                    ("sh_up", L.sh_up), ("sh_down", L.sh_down)):
        n = t.numel() // 144
        for first in [0] + list(rng.integers(0, n - 64, 3)):
            dev = t.view(-1, 144)[int(first):int(first) + 64].cpu().numpy()
            want = synth.law2_blocks(q4k.synth_blocks(4, stream_id(1, KIND_OF[kind]), int(first), 64))
            assert np.array_equal(dev, want), (kind, first)


@pytest.mark.parametrize("T", [1, 4, 12])
def test_law2_stack_teacher_forced(cuda, engine_law2, T):
    import torch
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import moe, synth
    from b200moe.engine import DeviceEngine
    resid = torch.from_numpy(bf16_bits_to_f32(synth.tokens(4, T, stream=90)).copy()).to(cuda)
    for l in range(N_LAYERS):
        before = resid.cpu().numpy().copy()
        ids = torch.empty((1, T, 8), dtype=torch.int32, device=cuda)
        moe.moe_stack(resid, DeviceEngine([engine_law2.layers[l]]), ids_out=ids, check=True)
        after = resid.cpu().numpy()
        Lh = host_layer2(4, l)
        xn = OM.rmsnorm(before)
        r = OM.router(xn, Lh.wg)
        got_ids = ids.cpu().numpy().reshape(T, 8)
        assert (got_ids == r["ids"]).all(), l
        ref = before.astype(np.float64) + OM.moe_block_f64(xn, Lh, r["ids"], r["w_bf16"])["out"]
        c = OM.compare(after, ref)
        distinct = len(np.unique(got_ids))
        rms = float(np.sqrt((after.astype(np.float64) ** 2).mean()))
        cos = float(np.corrcoef(xn)[np.triu_indices(T, 1)].max()) if T > 1 else 0.0
        print("law 2, T=%d, layer %d: distinct experts %d, resid rms %.3f, max token cosine %.3f, rel-L2 %.2e"
              % (T, l, distinct, rms, cos, c["rel_l2"]))
        assert c["rel_l2"] < 1e-5, (l, c)
        assert np.isfinite(after).all() and 0.05 < rms < 20.0, (l, rms)
        if T > 1:
            assert cos < 0.6 and distinct >= 4 * T, (l, cos, distinct)
