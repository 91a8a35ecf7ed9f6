"""Q5_K / Q6_K / Q8_0 restatements (oracle/kquants.py) against the reference's own decoders.

tests/golden/kquant_dequant.npz holds seeded and edge-case blocks of each format decoded by the
reference's tools/gguf_reader.py:dequant (checked identical to tools/gguf_fast_dequant.py:
dequant_np when the fixture was made). Bar: bit-exact f32 (NaN positions equal).
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden", "kquant_dequant.npz")


@pytest.mark.parametrize("tname", ["Q5_K", "Q6_K", "Q8_0"])
def test_restatement_matches_reference_decoder(tname):
    from oracle import kquants as KQ
    g = np.load(GOLD)
    mine = KQ.dequant(g[tname + "_blocks"], tname).view(np.uint32)
    ref = g[tname + "_ref_f32_bits"]
    both_nan = np.isnan(mine.view(np.float32)) & np.isnan(ref.view(np.float32))
    assert mine.shape == ref.shape and ((mine == ref) | both_nan).all()


def test_q6k_layout_known_answer():
    """One Q6_K block built by hand: element e gets q = e % 64 through the documented bit
    layout; d = 0.5, scale[e >> 4] = (e >> 4) - 8 -> value 0.5 * ((e >> 4) - 8) * (e % 64 - 32)."""
    from oracle import kquants as KQ
    raw = np.zeros(210, dtype=np.uint8)
    for e in range(256):
        q = e % 64
        g, k, l = e >> 7, (e >> 5) & 3, e & 31
        raw[64 * g + 32 * (k & 1) + l] |= (q & 15) << (4 * (k >> 1))
        raw[128 + 32 * g + l] |= (q >> 4) << (2 * k)
    raw[192:208] = (np.arange(16) - 8).astype(np.int8).view(np.uint8)
    raw[208:210] = np.array([0.5], dtype=np.float16).view(np.uint8)
    want = np.array([0.5 * ((e >> 4) - 8) * (e % 64 - 32) for e in range(256)], dtype=np.float32)
    assert np.array_equal(KQ.dequant_q6_k(raw), want)


def test_q5k_fifth_bit_known_answer():
    """One Q5_K block: d = 1, dmin = 0, every scale 1, all low nibbles 0, qh[l] = 0xFF -> every
    element is 16 (the fifth bit alone)."""
    from oracle import kquants as KQ, q4k
    raw = np.zeros(176, dtype=np.uint8)
    raw[0:2] = np.array([1.0], dtype=np.float16).view(np.uint8)
    raw[4:16] = q4k.pack_scale_min(np.ones(8, dtype=np.int64), np.zeros(8, dtype=np.int64))[0]
    raw[16:48] = 0xFF
    assert np.array_equal(KQ.dequant_q5_k(raw), np.full(256, 16.0, dtype=np.float32))


def test_host_layer_decodes_typed_kinds():
    """HostLayer with block types (the published file's down Q5_K / Q6_K, shared Q8_0) serves
    each kind's matrix through the pinned decoders, at the kind's own block count."""
    from oracle import kquants
    from oracle.moe import HostLayer
    H, I = 2048, 512
    blk = {"down": kquants.random_blocks("Q6_K", 3 * H * I // 256, 5),
           "sh_gate": kquants.random_blocks("Q8_0", I * H // 32, 6)}
    L = HostLayer(lambda k, f, n: blk[k][f:f + n], np.zeros(256 * H, np.uint16), np.zeros(H, np.uint16),
                  types={"down": "Q6_K", "sh_gate": "Q8_0"})
    per = H * I // 256
    assert np.array_equal(L.matrix("down", 2), kquants.dequant_q6_k(blk["down"][2 * per:3 * per]).reshape(H, I))
    assert np.array_equal(L.matrix("sh_gate"), kquants.dequant_q8_0(blk["sh_gate"]).reshape(I, H))
