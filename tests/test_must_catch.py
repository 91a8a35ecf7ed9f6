"""The must-catch set (the reference's injection tables: tools/gguf_reader.py:211,
prototype/q4k_dequant/q4k_dequant_kernels.h:125-142, speccheck/selftest_moe.py:57-67,
specification/10-reference-dumps-and-gates.md:90-108), planted in the ORACLE on the CPU: each
mistake a device path could make is shown to move the block output past the parity bars the GPU
tests apply (decode: rel-L2 1e-5; prefill: rel-L2 1e-3), or to break a bit-exact check, so a
kernel carrying it cannot pass. The correct oracle is the reference point throughout."""
import numpy as np
import pytest

from conftest import host_layer
from oracle import moe as OM
from oracle import q4k
from oracle.bf16 import bf16_bits_to_f32
from oracle.moe import HostLayer

DECODE_BAR, PREFILL_BAR = 1e-5, 1e-3
T = 4


@pytest.fixture(scope="module")
def case():
    import __graft_entry__ as G
    G.load_package()
    from b200moe import synth
    L = host_layer(0, 0)
    x = bf16_bits_to_f32(synth.tokens(0, T, stream=1))
    r = OM.router(x, L.wg)
    good = OM.moe_block_f64(x, L, r["ids"], r["w_bf16"])["out"]
    return L, x, r, good


def _planted(L, block_fn=None, matrix_fn=None):
    """L with a mistake in how its bytes are served (block_fn) or decoded (matrix_fn)."""
    P = HostLayer(block_fn or L._block_fn, L.wg, L.wsg, L.bias, L.types, L.norm_w)
    if matrix_fn is not None:
        P.matrix = lambda kind, e=0: matrix_fn(kind, e, lambda k, ee=0: HostLayer.matrix(P, k, ee))
    return P


def _swap_subblock_scales(L):
    def blocks(kind, first, n):
        raw = np.array(L._block_fn(kind, first, n), dtype=np.uint8, copy=True)
        sc, m = q4k.scale_min(np.ascontiguousarray(raw[:, 4:16]))
        sc = sc[:, [1, 0, 3, 2, 5, 4, 7, 6]]  # each sub-block reads its neighbour's scale
        raw[:, 4:16] = q4k.pack_scale_min(sc, m)
        return raw
    return _planted(L, block_fn=blocks)


def _drop_min(L):
    def blocks(kind, first, n):
        raw = np.array(L._block_fn(kind, first, n), dtype=np.uint8, copy=True)
        raw[:, 2:4] = 0  # dmin = +0: the -dmin*m term vanishes
        return raw
    return _planted(L, block_fn=blocks)


def _block_off_by_one(L):
    return _planted(L, block_fn=lambda kind, first, n: L._block_fn(kind, first + 1, n))


def _gate_up_swap(L):
    swap = {"gate": "up", "up": "gate", "sh_gate": "sh_up", "sh_up": "sh_gate"}
    return _planted(L, matrix_fn=lambda kind, e, base: base(swap.get(kind, kind), e))


def _transposed_down(L):
    def matrix(kind, e, base):
        w = base(kind, e)
        return w.reshape(w.shape[1], w.shape[0]).T if kind.endswith("down") else w
    return _planted(L, matrix_fn=matrix)


def _wrong_expert(L):
    return _planted(L, matrix_fn=lambda kind, e, base: base(kind, (e + 1) % 256 if not kind.startswith("sh_") else e))


@pytest.mark.parametrize("name,plant", [
    ("wrong sub-block scale", _swap_subblock_scales),
    ("dropped min", _drop_min),
    ("block off by one", _block_off_by_one),
    ("gate/up swap", _gate_up_swap),
    ("transposed down stack", _transposed_down),
    ("wrong expert index", _wrong_expert),
])
def test_planted_mistake_fails_the_bars(case, name, plant):
    """Each moves the output by rel-L2 >= 5e-2 here: tenfold past the looser prefill bar, so
    both the prefill and the decode parity tests would fail."""
    L, x, r, good = case
    bad = OM.moe_block_f64(x, plant(L), r["ids"], r["w_bf16"])["out"]
    c = OM.compare(bad, good)
    assert c["rel_l2"] > 10 * PREFILL_BAR, (name, c)


def test_dequant_level_mistakes_break_bit_exactness():
    """The dequant entry points are held bit-exact; the sub-block, min and offset mistakes each
    change most of a synthetic expert's values."""
    L = host_layer(0, 0)
    good = L.matrix("down", 3)
    for plant in (_swap_subblock_scales, _drop_min, _block_off_by_one):
        bad = plant(L).matrix("down", 3)
        assert np.count_nonzero(bad != good) > 0.5 * good.size, plant.__name__


def test_cast_after_breaks_the_r5_weights(case):
    """Multiplying by the f32 renormalised weight instead of its bf16 cast (cast-after) shows in
    the R5 weights, which the router tests compare bit for bit, and moves the output past the
    decode bar."""
    L, x, r, good = case
    from oracle.bf16 import f32_to_bf16_bits
    w_f32 = r["w_f32"].astype(np.float32)
    assert (f32_to_bf16_bits(w_f32) == r["w_bf16"]).all()          # the cast the kernels apply
    assert (bf16_bits_to_f32(r["w_bf16"]) != w_f32).mean() > 0.9    # what cast-after would use instead
    exp = OM.moe_block_f64(x, L, r["ids"], r["w_bf16"])
    routed_after = np.zeros_like(exp["routed"])
    for t in range(T):
        for k in range(8):
            routed_after[t] += exp["expert_raw"][t, k] * float(w_f32[t, k])
    c = OM.compare(routed_after + exp["shared_out"], good)
    assert c["rel_l2"] > DECODE_BAR, c


def test_rank_order_accumulation_is_below_the_output_bars(case):
    """Summing the weighted expert outputs in rank order instead of ascending expert id changes
    an f32 combine only in its last bits -- below every output bar, so no output comparison
    pins the order. (The reference pins it through a bf16 accumulator, where the order shows.)
    Recorded here so the limit of the output bars is explicit: the ascending order is the
    declared order of every combine in the kernels, and a stage-level bit-exact check of it is
    listed as next work."""
    L, x, r, good = case
    exp = OM.moe_block_f64(x, L, r["ids"], r["w_bf16"])
    raw = exp["expert_raw"].astype(np.float32)
    w = bf16_bits_to_f32(r["w_bf16"]).astype(np.float32)
    asc = np.zeros((T, raw.shape[-1]), np.float32)
    rank = np.zeros_like(asc)
    for t in range(T):
        for k in np.argsort(r["ids"][t], kind="stable"):
            asc[t] = asc[t] + raw[t, k] * w[t, k]
        for k in range(8):
            rank[t] = rank[t] + raw[t, k] * w[t, k]
    c = OM.compare(rank, asc)
    assert 0 < c["rel_l2"] < DECODE_BAR, c
