"""Seeded synthetic inputs for the BASELINE configurations (host side).

Q4_K expert weights are generated ON THE DEVICE by ``b200moe_synth_q4k`` (counter-based
splitmix64, field law in ``oracle/q4k.py:synth_blocks`` which mirrors it bit for bit), so a
40-layer stack (~18 GB) needs no host copy. The bf16 tensors (router W_g, shared gate w_sg,
token activations) are small and come from numpy's PCG64 normal generator, keyed by
(seed, tag), then rounded to bf16 (RNE):

* router W_g  [256, 2048] ~ N(0, 0.02)            tag (layer, 10)
* w_sg        [2048]      ~ N(0, 0.02)            tag (layer, 11)  -- law not given by the
                                                  baseline; chosen equal to W_g's
* tokens x    [T, 2048]   ~ N(0, 1) / sqrt(2048)  tag (1000 + stream,)
* Zipf bias   [256] f32   = tau * ln(p_rank(e)), p_r ~ r^-1.1 over a seeded permutation,
                          tag (layer, 12); tau calibrated so per-expert selection
                          frequency tracks Zipf(1.1) (config 2)
"""
from __future__ import annotations

import numpy as np

from .geometry import E, H

ZIPF_S = 1.1
ZIPF_TAU = 0.0125   # calibrated by zipf_calibrate(): L1 0.37 to Zipf(1.1), top-8 caps a share at 1/8


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    out = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    out[np.isnan(a)] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _normal_bf16(seed: int, tag: tuple, n: int, std: float) -> np.ndarray:
    rng = np.random.default_rng([int(seed), *[int(t) for t in tag]])
    v = rng.standard_normal(n, dtype=np.float32) * np.float32(std)
    return f32_to_bf16_bits(v)


def router_w(seed: int, layer: int) -> np.ndarray:
    return _normal_bf16(seed, (layer, 10), E * H, 0.02).reshape(E, H)


def shared_gate_w(seed: int, layer: int) -> np.ndarray:
    return _normal_bf16(seed, (layer, 11), H, 0.02)


def tokens(seed: int, T: int, stream: int = 0) -> np.ndarray:
    """[T, 2048] bf16 bits ~ N(0,1)/sqrt(2048) (an RMSNorm output's scale)."""
    return _normal_bf16(seed, (1000 + stream,), T * H, 1.0 / np.sqrt(H)).reshape(T, H)


def zipf_bias(seed: int, layer: int, tau: float = ZIPF_TAU, s: float = ZIPF_S) -> np.ndarray:
    rng = np.random.default_rng([int(seed), int(layer), 12])
    perm = rng.permutation(E)                    # perm[r] = expert holding rank r
    p = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** s
    p /= p.sum()
    bias = np.empty(E, dtype=np.float32)
    bias[perm] = (tau * np.log(p)).astype(np.float32)
    return bias - bias.max()


def zipf_calibrate(seed: int = 2, n_tok: int = 2048, taus=None) -> dict:
    """Pick tau so the per-expert selection frequency best matches Zipf(s) (L1 distance of the
    normalised selection histograms, sorted by rank). Host numpy f32; the calibration only
    sets a workload constant and needs no bit-exact logits."""
    taus = taus if taus is not None else [0.005, 0.01, 0.015, 0.02, 0.025, 0.03, 0.04, 0.06]
    x = bf16_bits_to_f32(tokens(seed, n_tok, stream=7))
    wg = bf16_bits_to_f32(router_w(seed, 0))
    base = x @ wg.T
    p = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** ZIPF_S
    p /= p.sum()
    best = None
    for tau in taus:
        lg = base + zipf_bias(seed, 0, tau)[None, :]
        top = np.argsort(-lg, axis=1, kind="stable")[:, :8]
        cnt = np.bincount(top.reshape(-1), minlength=E).astype(np.float64)
        freq = np.sort(cnt)[::-1] / cnt.sum()
        d = float(np.abs(freq - p).sum())
        if best is None or d < best[1]:
            best = (tau, d)
    return dict(tau=best[0], l1=best[1])


# ---------------------------------------------------------------- a second, centred weight law
# Under the field law above every Q4_K weight (d sc q - dmin m) has a mean of about +1.2, so a
# stack of such layers is dominated by one common residual direction after a layer and routing
# collapses onto the same experts. The second law keeps the seeded blocks and scales each
# super-block's f16 d by 2^-6 and dmin by 2^-2 (one RNE rounding each), which centres the
# weights: the residual stays O(1) and routing stays diverse through the stack.
LAW2_D_SCALE = 2.0 ** -6
LAW2_DMIN_SCALE = 2.0 ** -2


def law2_blocks(blocks: np.ndarray) -> np.ndarray:
    """Host: a scaled copy of Q4_K blocks (uint8, 144 bytes each)."""
    b = np.array(blocks, dtype=np.uint8, copy=True).reshape(-1, 144)
    h = b[:, 0:4].copy().view(np.float16).reshape(-1, 2)
    h[:, 0] = (h[:, 0] * np.float16(LAW2_D_SCALE)).astype(np.float16)
    h[:, 1] = (h[:, 1] * np.float16(LAW2_DMIN_SCALE)).astype(np.float16)
    b[:, 0:4] = h.view(np.uint8).reshape(-1, 4)
    return b


def law2_blocks_(t) -> None:
    """Device: the same scaling in place on a torch uint8 tensor of Q4_K blocks (the same bytes
    as law2_blocks: both round the exact product to f16 once, to nearest even)."""
    import torch
    b = t.view(-1, 144)
    h = b[:, 0:4].contiguous().view(torch.float16)
    h[:, 0] *= LAW2_D_SCALE
    h[:, 1] *= LAW2_DMIN_SCALE
    b[:, 0:4] = h.view(torch.uint8)
