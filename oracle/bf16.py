"""bf16 / f16 bit helpers for the oracle (test infrastructure only).

bf16 is the upper half of an IEEE binary32; conversion from f32 is round-to-nearest-even
(what ``torch.Tensor.to(torch.bfloat16)`` does and what the reference's R1/R5 casts use,
``engine/m3_forward.py:443,446``). NaN inputs map to the canonical quiet NaN 0x7FC0.
"""
import numpy as np


def f32_to_bf16_bits(a) -> np.ndarray:
    """Round f32 values to bf16 (RNE); returns uint16 bit patterns."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)
    nan = np.isnan(a)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(np.asarray(b, dtype=np.uint16))
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(a) -> np.ndarray:
    """f32 -> bf16 -> f32 (the value after an RNE cast)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))
