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
    Recorded here so the limit of the output bars is explicit; the order itself is pinned bit
    for bit at the stage level instead (tests/test_gpu_combine_order.py: routed_sum equals the
    ascending-id fold and differs from the rank-order one)."""
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


# ---------------------------------------------------------------------------------------------
# The three-arm discipline of the reference's self-test (speccheck/selftest_moe.py:8-28, its
# injection -> affected-stage table :57-67): per injection, the stages it must change (caught)
# and the stages that must stay bit-identical (kept).
#   honest  -- every injection changes its caught stages and no kept stage;
#   stub    -- with the difference predicate forced to "no difference", every catch is lost
#              (the checks are not vacuous: they rest on the comparison);
#   crossed -- a table that wrongly lists a changed stage as kept is flagged.
STAGES = ("ids", "w", "expert_raw", "shared_raw", "shared_gate_prob", "routed", "out")


def _stages(L, x, ids, w):
    """Stage values of the block with routing (ids, w: the weights applied, f64)."""
    from oracle.bf16 import f32_to_bf16_bits
    d = OM.moe_block_f64(x, L, ids, f32_to_bf16_bits(np.asarray(w, np.float32)))
    routed = np.einsum("tkh,tk->th", d["expert_raw"], np.asarray(w, np.float64))
    return dict(ids=np.asarray(ids), w=np.asarray(w, np.float64), expert_raw=d["expert_raw"],
                shared_raw=d["shared_raw"], shared_gate_prob=d["shared_gate_prob"], routed=routed,
                out=routed + d["shared_out"])


def _route_bf16_softmax(r):
    """Top-8 and renormalisation over the softmax probabilities rounded to bf16."""
    from oracle.bf16 import bf16_bits_to_f32 as b2f, f32_to_bf16_bits as f2b
    pb = b2f(f2b(r["probs"])).astype(np.float64)
    ids = np.stack([np.lexsort((np.arange(pb.shape[1]), -row))[:8] for row in pb]).astype(np.int32)
    p = np.take_along_axis(pb, ids, 1)
    return ids, b2f(f2b((p / p.sum(1, keepdims=True)).astype(np.float32)))


ROUTED = {"expert_raw", "routed", "out"}
WEIGHTS = {"w", "routed", "out"}


def _table(L, r):
    """name -> (layer, ids, w applied, caught stages, kept stages)."""
    from oracle.bf16 import bf16_bits_to_f32 as b2f, f32_to_bf16_bits as f2b
    ids, w = r["ids"], b2f(r["w_bf16"])
    swap_routed = {"gate": "up", "up": "gate"}
    swap_shared = {"sh_gate": "sh_up", "sh_up": "sh_gate"}
    p_top = np.take_along_axis(r["probs"], r["ids"].astype(np.int64), 1)
    sb_ids, sb_w = _route_bf16_softmax(r)
    every = set(STAGES)
    t = {
        "wrong expert index": (_wrong_expert(L), ids, w, ROUTED),
        "gate/up swap": (_planted(L, matrix_fn=lambda k, e, base: base(swap_routed.get(k, k), e)), ids, w, ROUTED),
        "transposed expert stack": (_planted(L, matrix_fn=lambda k, e, base: (
            lambda m: m.reshape(m.shape[1], m.shape[0]).T if k == "down" else m)(base(k, e))), ids, w, ROUTED),
        "shared gate/up swap": (_planted(L, matrix_fn=lambda k, e, base: base(swap_shared.get(k, k), e)), ids, w,
                                {"shared_raw", "out"}),
        "renorm omitted": (L, ids, b2f(f2b(p_top)), WEIGHTS),
        "cast after multiply": (L, ids, r["w_f32"], WEIGHTS),
        "softmax in bf16": (L, sb_ids, sb_w, WEIGHTS),
        "wrong sub-block scale": (_swap_subblock_scales(L), ids, w, ROUTED | {"shared_raw"}),
        "dropped min": (_drop_min(L), ids, w, ROUTED | {"shared_raw"}),
        "block off by one": (_block_off_by_one(L), ids, w, ROUTED | {"shared_raw"}),
    }
    kept_always = {"softmax in bf16": {"shared_raw", "shared_gate_prob"}}  # its ids may move with the ties
    return {n: (Lp, i, ww, caught, kept_always.get(n, every - caught)) for n, (Lp, i, ww, caught) in t.items()}


def _differs(a, b):
    return not np.array_equal(np.asarray(a), np.asarray(b))


@pytest.fixture(scope="module")
def arms(case):
    L, x, r, _ = case
    from oracle.bf16 import bf16_bits_to_f32 as b2f
    good = _stages(L, x, r["ids"], b2f(r["w_bf16"]))
    runs = {n: (_stages(Lp, x, i, ww), caught, kept) for n, (Lp, i, ww, caught, kept) in _table(L, r).items()}
    return good, runs


def _verdict(good, bad, caught, kept, differs):
    missed = [s for s in sorted(caught) if not differs(good[s], bad[s])]
    breached = [s for s in sorted(kept) if differs(good[s], bad[s])]
    return missed, breached


def test_honest_arm(arms):
    good, runs = arms
    for name, (bad, caught, kept) in runs.items():
        assert _verdict(good, bad, caught, kept, _differs) == ([], []), name


def test_stub_arm_loses_every_catch(arms):
    good, runs = arms
    for name, (bad, caught, kept) in runs.items():
        missed, breached = _verdict(good, bad, caught, kept, lambda a, b: False)
        assert missed == sorted(caught) and breached == [], name


def test_crossed_arm_flags_a_misdeclared_stage(arms):
    good, runs = arms
    for name, (bad, caught, kept) in runs.items():
        stage = sorted(caught)[0]                      # declare one changed stage as kept
        missed, breached = _verdict(good, bad, caught - {stage}, kept | {stage}, _differs)
        assert missed == [] and breached == [stage], name
