"""Q5_K, Q6_K and Q8_0 restatements (test infrastructure only).

The published Qwen3.6-35B-A3B Q4_K_M file mixes block formats: most expert down matrices are
Q5_K, a few Q6_K, and the shared expert is Q8_0. The reference decodes them in
``tools/gguf_reader.py:238-333`` (scalar, f64) and ``tools/gguf_fast_dequant.py:109-150``
(numpy, f64, one rounding to f32 at the end); both transcribe llama.cpp's
``dequantize_row_q5_K / q6_K / q8_0`` (llama.cpp d327bf1f0780f87b8c01b367b61853b0c291d7c4,
not vendored in the reference). This file restates the same layouts:

* Q8_0, 34 B per 32 weights: f16 d, then 32 int8 q; value = d * q.
* Q5_K, 176 B per 256 weights: f16 d, f16 dmin, 12 scale bytes (the Q4_K packing of eight
  6-bit scales and mins), 32 bytes qh (the fifth bits), 128 bytes qs (low four bits).
  Element e: sub-block j = e >> 5; byte 48 + 32*(e >> 6) + (e & 31) of qs, low nibble when j
  is even, high when odd; fifth bit = bit j of qh[e & 31]; value = (d*sc[j])*q - dmin*m[j].
* Q6_K, 210 B per 256 weights: 128 bytes ql, 64 bytes qh, 16 int8 scales, f16 d (LAST).
  Group g = e >> 7, k = (e >> 5) & 3, l = e & 31: low four bits = ql[64g + 32(k & 1) + l]
  shifted right by 4 when k >= 2; high two bits = (qh[32g + l] >> 2k) & 3; scale index
  8g + 2k + (l >> 4) = e >> 4; value = (d*sc)*(q - 32).

Every product is exact in f32 (Q8_0 <= 19 significant bits, Q5_K <= 22, Q6_K <= 23), so the
reference's f64 route rounds exactly once (Q5_K: at the subtraction; Q6_K, Q8_0: not at all)
and these f32 expressions reproduce it bit for bit. Pinned against the reference's own
decoders by ``tests/golden/kquant_dequant.npz`` (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import numpy as np

from . import q4k

QK_K = 256
BLOCK_BYTES = {"Q8_0": 34, "Q5_K": 176, "Q6_K": 210, "Q4_K": 144}
BLOCK_ELTS = {"Q8_0": 32, "Q5_K": 256, "Q6_K": 256, "Q4_K": 256}


def _blocks(buf, tname: str, nblocks: int | None) -> np.ndarray:
    b = np.frombuffer(bytes(buf) if not isinstance(buf, np.ndarray) else buf.tobytes(), dtype=np.uint8)
    bb = BLOCK_BYTES[tname]
    n = b.size // bb if nblocks is None else int(nblocks)
    if b.size < n * bb:
        raise ValueError("short buffer: %d %s blocks need %d B, got %d" % (n, tname, n * bb, b.size))
    return b[: n * bb].reshape(n, bb)


def _f16(raw: np.ndarray, col: int) -> np.ndarray:
    return np.ascontiguousarray(raw[:, col:col + 2]).view("<f2").astype(np.float32).reshape(-1)


def dequant_q8_0(buf, nblocks: int | None = None) -> np.ndarray:
    raw = _blocks(buf, "Q8_0", nblocks)
    d = _f16(raw, 0)
    q = np.ascontiguousarray(raw[:, 2:34]).view(np.int8).astype(np.float32)
    return (d[:, None] * q).reshape(-1)


def dequant_q5_k(buf, nblocks: int | None = None) -> np.ndarray:
    raw = _blocks(buf, "Q5_K", nblocks)
    nb = raw.shape[0]
    d, dmin = _f16(raw, 0), _f16(raw, 2)
    sc, m = q4k.scale_min(np.ascontiguousarray(raw[:, 4:16]))          # [nb, 8] each
    qh = raw[:, 16:48]                                                  # [nb, 32]
    qs = raw[:, 48:176].reshape(nb, 4, 32)                              # byte 32g + l
    out = np.empty((nb, 8, 32), dtype=np.float32)
    for j in range(8):
        g = j >> 1
        low = (qs[:, g, :] >> (4 * (j & 1))) & 0xF
        hi = (qh >> j) & 1
        q = (low | (hi << 4)).astype(np.float32)
        s = d * sc[:, j].astype(np.float32)                             # exact
        mm = dmin * m[:, j].astype(np.float32)                          # exact
        out[:, j, :] = s[:, None] * q - mm[:, None]                     # one rounding
    return out.reshape(-1)


def dequant_q6_k(buf, nblocks: int | None = None) -> np.ndarray:
    raw = _blocks(buf, "Q6_K", nblocks)
    nb = raw.shape[0]
    ql = raw[:, 0:128]
    qh = raw[:, 128:192]
    sc = np.ascontiguousarray(raw[:, 192:208]).view(np.int8).astype(np.float32)   # [nb, 16]
    d = _f16(raw, 208)
    out = np.empty((nb, 2, 4, 32), dtype=np.float32)
    for g in range(2):
        for k in range(4):
            low = (ql[:, 64 * g + 32 * (k & 1): 64 * g + 32 * (k & 1) + 32] >> (4 * (k >> 1))) & 0xF
            hi = (qh[:, 32 * g: 32 * g + 32] >> (2 * k)) & 3
            q = (low | (hi << 4)).astype(np.float32) - 32.0
            s = np.repeat((d[:, None] * sc[:, 8 * g + 2 * k: 8 * g + 2 * k + 2]), 16, axis=1)  # exact
            out[:, g, k, :] = s * q                                                        # exact
    return out.reshape(-1)


def dequant(buf, tname: str, nblocks: int | None = None) -> np.ndarray:
    """f32 values of ``nblocks`` blocks of ``tname`` (Q4_K, Q5_K, Q6_K or Q8_0)."""
    if tname == "Q4_K":
        return q4k.dequant(buf, nblocks)
    fn = {"Q5_K": dequant_q5_k, "Q6_K": dequant_q6_k, "Q8_0": dequant_q8_0}.get(tname)
    if fn is None:
        raise NotImplementedError("no decoder for %r" % tname)
    return fn(buf, nblocks)


def random_blocks(tname: str, n: int, seed: int) -> np.ndarray:
    """``n`` seeded blocks with finite, normal f16 scale fields (every other byte random)."""
    rng = np.random.default_rng(seed)
    bb = BLOCK_BYTES[tname]
    raw = rng.integers(0, 256, size=(n, bb), dtype=np.uint8)
    cols = {"Q8_0": (0,), "Q5_K": (0, 2), "Q6_K": (208,)}[tname]
    for c in cols:
        h = rng.uniform(1e-4, 2e-2, size=n).astype(np.float16)
        h = np.where(rng.random(n) < 0.2, -h, h).astype(np.float16)
        raw[:, c:c + 2] = h.view(np.uint8).reshape(n, 2)
    return raw
