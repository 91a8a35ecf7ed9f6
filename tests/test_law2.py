"""The second, centred weight law of the synthetic stack (synth.law2_blocks / law2_blocks_), on CPU:
only each super-block's f16 d and dmin change (by 2^-6 and 2^-2, one RNE rounding each), the torch
in-place form gives the numpy form's bytes, and the law does what it is for -- the dequantised
weights are centred (the BASELINE field law's mean is about +1.2)."""
import numpy as np

from oracle import q4k


def test_law2_scales_only_d_and_dmin():
    from b200moe import synth
    b = q4k.synth_blocks(4, 3, 0, 4096)
    c = synth.law2_blocks(b)
    assert np.array_equal(b[:, 4:], c[:, 4:])
    d0 = b[:, 0:4].copy().view(np.float16).astype(np.float64).reshape(-1, 2)
    d1 = c[:, 0:4].copy().view(np.float16).astype(np.float64).reshape(-1, 2)
    normal = d0[:, 0] * 2.0 ** -6 >= 2.0 ** -14          # no subnormal rounding: exact
    assert np.array_equal(d1[normal, 0], d0[normal, 0] * 2.0 ** -6)
    assert np.array_equal(d1[:, 1][d0[:, 1] * 0.25 >= 2.0 ** -14], (d0[:, 1] * 0.25)[d0[:, 1] * 0.25 >= 2.0 ** -14])
    # where the scaled value is subnormal it is the round-to-nearest-even f16 of the exact product
    assert np.array_equal(d1[:, 0], (d0[:, 0] * 2.0 ** -6).astype(np.float16).astype(np.float64))


def test_law2_torch_matches_numpy():
    import torch
    from b200moe import synth
    b = q4k.synth_blocks(4, 7, 0, 2048)
    t = torch.from_numpy(b.reshape(-1).copy())
    synth.law2_blocks_(t)
    assert np.array_equal(t.numpy().reshape(-1, 144), synth.law2_blocks(b))


def test_law2_centres_the_weights():
    from b200moe import synth
    b = q4k.synth_blocks(4, 11, 0, 2048)
    w1 = q4k.dequant(b.tobytes()).astype(np.float64)
    w2 = q4k.dequant(synth.law2_blocks(b).tobytes()).astype(np.float64)
    assert w1.mean() > 0.5                                # the BASELINE law: strongly positive
    assert abs(w2.mean()) < 0.1 * w2.std()                # law 2: centred
