"""GGUF Q4_K restatement and synthetic-block mirror (test infrastructure only).

Block layout (``block_q4_K``; reference ``prototype/q4k_dequant/q4k_dequant_kernels.h:94-103``
and ``tools/gguf_reader.py:29-45``): 144 bytes per 256 weights::

    bytes 0..1    f16 d       (super-block scale)
    bytes 2..3    f16 dmin    (super-block min scale; the stored min is a MAGNITUDE)
    bytes 4..15   12 bytes holding 8 six-bit scales and 8 six-bit mins (get_scale_min_k4)
    bytes 16..143 128 bytes of 4-bit quants

Element e (0..255): sub-block j = e >> 5, byte 16 + 32*(e >> 6) + (e & 31), low nibble
when j is even, high nibble when j is odd; value = (d*sc[j])*q - dmin*m[j].

Every product in that expression is exact in f32 (<= 21 significant bits), so both the
reference's f64 route and an f32 route round exactly once, at the subtraction.
"""
from __future__ import annotations

import numpy as np

QK_K = 256
BLOCK_BYTES = 144

# ----------------------------------------------------------------------------------------
# get_scale_min_k4 and its inverse
# ----------------------------------------------------------------------------------------


def scale_min(scales: np.ndarray):
    """(sc[nb,8], m[nb,8]) as int64 from the 12 scale bytes [nb,12].

    Restates ``tools/gguf_reader.py:165-176`` (``qk_scale_min``) and
    ``tools/gguf_fast_dequant.py:75-84`` (``_scale_min_qk``)::

        j < 4 : sc = q[j] & 63                       m = q[j+4] & 63
        j >= 4: sc = (q[j+4] & 0xF) | ((q[j-4] >> 6) << 4)
                m  = (q[j+4] >> 4)  | ((q[j]   >> 6) << 4)
    """
    q = np.asarray(scales, dtype=np.uint8).reshape(-1, 12).astype(np.int64)
    sc = np.empty((q.shape[0], 8), dtype=np.int64)
    m = np.empty((q.shape[0], 8), dtype=np.int64)
    sc[:, 0:4] = q[:, 0:4] & 63
    m[:, 0:4] = q[:, 4:8] & 63
    sc[:, 4:8] = (q[:, 8:12] & 0xF) | ((q[:, 0:4] >> 6) << 4)
    m[:, 4:8] = (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)
    return sc, m


def pack_scale_min(sc, m) -> np.ndarray:
    """Inverse of :func:`scale_min`: 8 scales + 8 mins (0..63) -> 12 bytes.

    Same inverse as the reference's ``prototype/q4k_dequant/gate.py:322-337``
    (``pack_scale_min``); checked by round trip in the tests.
    """
    sc = np.asarray(sc, dtype=np.int64).reshape(-1, 8)
    m = np.asarray(m, dtype=np.int64).reshape(-1, 8)
    q = np.zeros((sc.shape[0], 12), dtype=np.int64)
    q[:, 0:4] |= sc[:, 0:4] & 63
    q[:, 4:8] |= m[:, 0:4] & 63
    q[:, 4:8] |= (m[:, 4:8] >> 4) << 6
    q[:, 0:4] |= ((sc[:, 4:8] >> 4) & 3) << 6
    q[:, 8:12] |= (sc[:, 4:8] & 15) | ((m[:, 4:8] & 15) << 4)
    return q.astype(np.uint8)


def build_block(d_bits: int, dmin_bits: int, sc, m, qs) -> bytes:
    """One 144-byte block from its fields (f16 bit patterns for d/dmin)."""
    raw = np.zeros(BLOCK_BYTES, dtype=np.uint8)
    raw[0:2] = np.array([d_bits], dtype="<u2").view(np.uint8)
    raw[2:4] = np.array([dmin_bits], dtype="<u2").view(np.uint8)
    raw[4:16] = pack_scale_min(sc, m)[0]
    raw[16:144] = np.asarray(qs, dtype=np.uint8)
    return raw.tobytes()


# ----------------------------------------------------------------------------------------
# dequant
# ----------------------------------------------------------------------------------------


def dequant(buf, nblocks: int | None = None) -> np.ndarray:
    """Q4_K bytes -> f32 values in stored element order.

    Restates ``tools/gguf_reader.py:248-267`` (``_deq_q4_k``) and the Q4_K branch of
    ``tools/gguf_fast_dequant.py:109-125``: the expression is evaluated in f64 (exact) and
    rounded once to f32. f16 NaN/Inf fields propagate as IEEE arithmetic dictates.
    """
    raw = np.frombuffer(bytes(buf) if not isinstance(buf, np.ndarray) else buf.tobytes(),
                        dtype=np.uint8)
    if nblocks is None:
        nblocks = raw.size // BLOCK_BYTES
    raw = raw[: nblocks * BLOCK_BYTES].reshape(nblocks, BLOCK_BYTES)
    d = np.ascontiguousarray(raw[:, 0:2]).view("<f2").astype(np.float64).reshape(-1, 1, 1, 1)
    dmin = np.ascontiguousarray(raw[:, 2:4]).view("<f2").astype(np.float64).reshape(-1, 1, 1, 1)
    sc, m = scale_min(raw[:, 4:16])
    qs = raw[:, 16:144].reshape(-1, 4, 32)
    q = np.stack([qs & 0xF, qs >> 4], axis=2).astype(np.float64)         # (nb, 4, 2, 32)
    sc = sc.reshape(-1, 4, 2, 1).astype(np.float64)
    m = m.reshape(-1, 4, 2, 1).astype(np.float64)
    with np.errstate(invalid="ignore", over="ignore"):
        vals = (d * sc) * q - dmin * m
    return vals.reshape(-1).astype(np.float32)


def dequant_drop_min(buf, nblocks: int | None = None) -> np.ndarray:
    """The ``q4k_drop_min`` misreading (``tools/gguf_reader.py:211-220`` INJECTIONS):
    value = d*sc*q without the min term. Used as a must-catch control in tests."""
    raw = np.frombuffer(bytes(buf), dtype=np.uint8)
    if nblocks is None:
        nblocks = raw.size // BLOCK_BYTES
    raw = raw[: nblocks * BLOCK_BYTES].reshape(nblocks, BLOCK_BYTES).copy()
    raw[:, 2:4] = 0
    return dequant(raw.tobytes(), nblocks)


# ----------------------------------------------------------------------------------------
# seeded synthetic blocks -- numpy mirror of the device generator (b200moe_synth_q4k)
# ----------------------------------------------------------------------------------------
GOLDEN = np.uint64(0x9E3779B97F4A7C15)
WORDS_PER_BLOCK = 19


def _mix64(z: np.ndarray) -> np.ndarray:
    """splitmix64's output function (Steele, Lea & Flood 2014)."""
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def stream_key(seed: int, stream: int) -> np.uint64:
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + GOLDEN * np.uint64(stream + 1)
    return _mix64(np.array([z], dtype=np.uint64))[0]


def synth_blocks(seed: int, stream: int, block0: int, nblocks: int) -> np.ndarray:
    """Blocks [block0, block0+nblocks) of synthetic stream ``stream`` -> uint8 [nblocks,144].

    Field law (the BASELINE config-0 law): f16 d ~ U(1e-3, 1e-2), f16 dmin ~ U(0, 5e-3),
    the 12 scale bytes uniformly random (get_scale_min_k4 is a bijection of the 96 bits, so
    every sc and m is U{0..63} and independent), every 4-bit quant U{0..15}.

    Word w of block b is ``mix64(key + GOLDEN*(19*b + w + 1))`` with
    ``key = mix64(seed + GOLDEN*(stream+1))``:
      w0 bits [0,24)  -> u_d,  d    = f16_rne(1e-3f + u_d * 2^-24 * 9e-3f)   (f32 mul, then add)
      w0 bits [32,56) -> u_m,  dmin = f16_rne(u_m * 2^-24 * 5e-3f)
      w1, w2[0:4]     -> the 12 scale bytes (little endian)
      w3 .. w18       -> the 128 quant bytes (little endian)
    """
    key = stream_key(seed, stream)
    b = np.arange(block0, block0 + nblocks, dtype=np.uint64)
    idx = b[:, None] * np.uint64(WORDS_PER_BLOCK) + np.arange(WORDS_PER_BLOCK, dtype=np.uint64)[None, :]
    with np.errstate(over="ignore"):
        words = _mix64(key + GOLDEN * (idx + np.uint64(1)))          # [nb, 19]
    out = np.empty((nblocks, BLOCK_BYTES), dtype=np.uint8)
    w0 = words[:, 0]
    u_d = (w0 & np.uint64(0xFFFFFF)).astype(np.float32) * np.float32(2.0 ** -24)
    u_m = ((w0 >> np.uint64(32)) & np.uint64(0xFFFFFF)).astype(np.float32) * np.float32(2.0 ** -24)
    d32 = np.float32(1e-3) + u_d * np.float32(9e-3)
    m32 = u_m * np.float32(5e-3)
    out[:, 0:2] = d32.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = m32.astype(np.float16).view(np.uint8).reshape(-1, 2)
    wb = np.ascontiguousarray(words.astype("<u8")).view(np.uint8).reshape(nblocks, WORDS_PER_BLOCK * 8)
    out[:, 4:16] = wb[:, 8:20]
    out[:, 16:144] = wb[:, 24:152]
    return out
