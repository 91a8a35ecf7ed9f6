"""The oracle pinned against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference's Python). CPU only."""
import hashlib

import numpy as np
import pytest

from conftest import golden, host_layer
from oracle import moe as OM
from oracle import q4k
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits


def same_bits(a, b):
    a = np.asarray(a, np.float32).view(np.uint32)
    b = np.asarray(b, np.float32).view(np.uint32)
    nan = ((a & 0x7FFFFFFF) > 0x7F800000) & ((b & 0x7FFFFFFF) > 0x7F800000)
    return (a == b) | nan


def test_dequant_numpy_bit_exact_vs_reference():
    g = golden("q4k_dequant.npz")
    got = q4k.dequant(g["blocks"].tobytes())
    assert same_bits(got, g["ref_f32_bits"].view(np.float32)).all()


def test_dequant_c_bit_exact_vs_reference():
    g = golden("q4k_dequant.npz")
    got = OM.dequant_c(g["blocks"])
    assert same_bits(got, g["ref_f32_bits"].view(np.float32)).all()


def test_known_answer_945():
    g = golden("q4k_dequant.npz")
    i = list(g["labels"]).index("kat945")
    v = q4k.dequant(g["blocks"][i].tobytes())
    assert np.count_nonzero(v) == 1 and v[33] == 945.0


def test_must_catch_drop_min_fires():
    """q4k_drop_min (tools/gguf_reader.py:211 INJECTIONS) must change synthetic blocks."""
    g = golden("q4k_dequant.npz")
    labels = list(g["labels"])
    syn = g["blocks"][[i for i, l in enumerate(labels) if l.startswith("synth_")]]
    good = q4k.dequant(syn.tobytes())
    bad = q4k.dequant_drop_min(syn.tobytes())
    assert np.count_nonzero(good != bad) > 0.9 * good.size


def test_pack_scale_min_round_trip():
    rng = np.random.default_rng(3)
    sc = rng.integers(0, 64, (100, 8))
    m = rng.integers(0, 64, (100, 8))
    sc2, m2 = q4k.scale_min(q4k.pack_scale_min(sc, m))
    assert (sc2 == sc).all() and (m2 == m).all()


def test_synth_field_law():
    b = q4k.synth_blocks(0, 3, 0, 4096)
    d = b[:, 0:2].copy().view("<f2").astype(np.float64).ravel()
    dm = b[:, 2:4].copy().view("<f2").astype(np.float64).ravel()
    assert (d >= 9.99e-4).all() and (d <= 1.00022e-2).all()   # f16 rounding of the U(1e-3,1e-2) bounds
    assert (dm >= 0).all() and (dm <= 5.0025e-3).all()
    sc, m = q4k.scale_min(b[:, 4:16])
    assert sc.min() == 0 and sc.max() == 63 and m.min() == 0 and m.max() == 63
    q = np.concatenate([b[:, 16:] & 15, b[:, 16:] >> 4])
    assert abs(q.mean() - 7.5) < 0.05
    # deterministic and position-keyed: a sub-range equals the slice of the full range
    assert (q4k.synth_blocks(0, 3, 100, 7) == b[100:107]).all()


def test_expf_error_bound():
    """The library's own exp (shared by the CUDA router) within 2 ulp of exp over softmax's range."""
    x = np.concatenate([np.linspace(-30, 0, 4001), -np.logspace(-8, 1.4, 500), [0.0, -1e-30]]).astype(np.float32)
    got = OM.expf(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(got - ref) / ulp) <= 2.0


def test_router_vs_reference():
    """Declared-order R1..R5 (oracle/c/oracle.c) against the reference's torch R1..R5.

    R1's f32 summation order differs from torch's, so a logit may move by one bf16 ulp;
    the selected ids must agree on every row whose 8th/9th probabilities are not tied,
    and the bf16 weights within one ulp."""
    g = golden("router_t64.npz")
    from b200moe import synth
    wg = synth.router_w(0, 0)
    assert hashlib.sha256(wg.tobytes()).hexdigest() == str(g["wg_sha256"])
    r = OM.router(bf16_bits_to_f32(g["x_bits"]), wg)
    dl = np.abs(r["logits"].astype(np.int32) - g["logits_bits"].astype(np.int32))
    assert dl.max() <= 1 and np.count_nonzero(dl) <= 0.01 * dl.size
    probs = g["probs"]
    srt = np.sort(probs, axis=1)[:, ::-1]
    tie = srt[:, 7] == srt[:, 8]
    for t in range(64):
        if not tie[t]:
            assert set(r["ids"][t]) == set(g["ids"][t]), t
            ours = dict(zip(r["ids"][t], r["w_bf16"][t].astype(np.int32)))
            theirs = dict(zip(g["ids"][t], g["wcast_bits"][t].astype(np.int32)))
            assert all(abs(ours[e] - theirs[e]) <= 1 for e in ours)


def test_moe_block_f64_vs_reference():
    """f64 restatement of m3_forward.moe_block vs the reference run on the same seeded weights."""
    g = golden("moe_block_t4.npz")
    L = host_layer(0, 0)
    x = bf16_bits_to_f32(g["x_bits"])
    r = OM.router(x, L.wg)
    ref_ids = g["ids"]
    ties = 0
    for t in range(4):
        if (r["ids"][t] != ref_ids[t]).any():
            # only an exact tie may differ: same rank position, equal bf16 logits
            k = np.nonzero(r["ids"][t] != ref_ids[t])[0]
            assert (r["logits"][t][r["ids"][t][k]] == r["logits"][t][ref_ids[t][k]]).all(), t
            ties += 1
    assert ties <= 1
    # tied experts have equal probabilities, hence equal R5 weights at the same rank
    w = r["w_bf16"]
    got = OM.moe_block_f64(x, L, ref_ids, w)["out"]
    c = OM.compare(got, g["out"])
    assert c["rel_l2"] < 2e-6 and c["max_abs_norm"] < 2e-6, c


def test_moe_block_port_vs_reference():
    """The torch-f32 port (the timed CPU baseline) reproduces the reference's output."""
    g = golden("moe_block_t4.npz")
    L = host_layer(0, 0)
    out, ids = OM.moe_block_port(bf16_bits_to_f32(g["x_bits"]), L, threads=4)
    assert (ids == g["ids"]).all()
    c = OM.compare(out, g["out"])
    assert c["rel_l2"] < 1e-6, c


def test_rmsnorm_vs_reference():
    g = golden("rmsnorm.npz")
    y = OM.rmsnorm(g["x"])
    ulp = np.spacing(np.abs(g["y"]).astype(np.float32))
    assert np.max(np.abs(y - g["y"]) / ulp) <= 2.0


def test_bf16_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, np.nan, 3.4e38, 1e-40], np.float32)
    import torch
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    ours = f32_to_bf16_bits(x)
    fin = ~np.isnan(x)
    assert (ours[fin] == ref[fin]).all()
    assert ((ours[~fin] & 0x7FFF) > 0x7F80).all()      # NaN stays NaN (payload not compared)
