"""The fixed-point arithmetic of the tensor-core Q4_K dots (csrc/imma.cuh), restated in numpy and
checked on the CPU.

The persistent single-token kernel and the grouped small-batch kernels compute each expert dot as
int8 MMAs: the vector v is scaled by 2^k, k = 21 - floor(log2 max|v|), rounded to integers
|n| <= 2^22 and split into three signed base-256 digits; each 32-element sub-block's integer sum
sum(q * n) is exact; the 6-bit scales multiply it in int32; d, dmin and 2^-k are applied in f32.
These tests pin what that arithmetic promises, independently of the GPU:
  * the digit split is exact and stays in range for every |n| <= 2^22 (and never overflows for
    any int32, whose garbage digits only ever meet a NaN scale);
  * the per-super-block int32 sums cannot overflow;
  * the dot differs from the exact (f64) dot of the same Q4_K row with the unrounded v by at most
    sum|w| * max|v| * 2^-22 (the rounding of v, with f32 combine headroom) -- in practice ~1e-7 of
    ||w|| ||v||, far inside the 1e-5 decode parity bar.
"""
import numpy as np
import pytest

from oracle import q4k


def digit_shift(mbits: int) -> int:
    if mbits == 0 or mbits >= 0x7F800000:
        return 0
    return min(21 - ((mbits >> 23) - 127), 126)


def digits3(n):
    """Vectorised digits3 (int64 arithmetic, the kernel's int32 ops have the same results)."""
    n = np.asarray(n, dtype=np.int64)
    d2 = n & 255
    d2 = d2 - ((d2 & 128) << 1)
    r = (n >> 8) + ((n >> 7) & 1)
    d1 = r & 255
    d1 = d1 - ((d1 & 128) << 1)
    d0 = (r >> 8) + ((r >> 7) & 1)
    return d0, d1, d2


def image(v: np.ndarray):
    """(n, k): the integer image of f32 vector v and its power-of-two shift."""
    v = np.asarray(v, dtype=np.float32)
    mbits = int((v.view(np.uint32) & 0x7FFFFFFF).max())
    k = digit_shift(mbits)
    n = np.rint((v * np.float32(2.0 ** k)).astype(np.float32)).astype(np.int64)
    return n, k


def q4k_fields(blocks: np.ndarray):
    """(d, dmin, sc[nb,8], m[nb,8], q[nb,256]) of raw Q4_K blocks [nb, 144]."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float64).reshape(-1)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float64).reshape(-1)
    sc, m = q4k.scale_min(b[:, 4:16])
    qs = b[:, 16:].astype(np.int64)
    q = np.empty((b.shape[0], 256), dtype=np.int64)
    for j in range(4):
        grp = qs[:, 32 * j:32 * j + 32]
        q[:, 64 * j:64 * j + 32] = grp & 15
        q[:, 64 * j + 32:64 * j + 64] = grp >> 4
    return d, dmin, sc, m, q


def digit_dot(blocks: np.ndarray, v: np.ndarray) -> float:
    """One Q4_K row (nb super-blocks) against v, the way the MMA path composes it."""
    d, dmin, sc, m, q = q4k_fields(blocks)
    n, k = image(v)
    d0, d1, d2 = digits3(n)
    nb = q.shape[0]
    total = 0.0
    for b in range(nb):
        qb = q[b].reshape(8, 32)
        ia = [0, 0, 0]
        for pl, dg in enumerate((d0, d1, d2)):
            sub = (qb * dg[256 * b:256 * b + 256].reshape(8, 32)).sum(1)  # exact per sub-block
            assert np.abs(sub).max() <= 32 * 15 * 128
            acc = int((sc[b] * sub).sum())
            assert -2 ** 31 <= acc < 2 ** 31  # the int32 super-block accumulator
            ia[pl] = acc
        sx = n[256 * b:256 * b + 256].reshape(8, 32).sum(1)
        total += d[b] * (65536.0 * ia[0] + 256.0 * ia[1] + ia[2]) - dmin[b] * float((m[b] * sx).sum())
    return total * 2.0 ** -k


def test_digits_exact_and_in_range():
    rng = np.random.default_rng(0)
    edge = np.array([0, 1, -1, 127, 128, -128, -129, 255, 256, -256, 32767, -32768, 65535, 65536,
                     2 ** 22, -2 ** 22, 2 ** 22 - 1, -(2 ** 22) + 1], dtype=np.int64)
    n = np.concatenate([edge, rng.integers(-2 ** 22, 2 ** 22 + 1, 200000)])
    d0, d1, d2 = digits3(n)
    assert np.array_equal(65536 * d0 + 256 * d1 + d2, n)
    assert d1.min() >= -128 and d1.max() <= 127 and d2.min() >= -128 and d2.max() <= 127
    assert np.abs(d0).max() <= 64
    # any int32 (the garbage of a non-finite vector): no overflow, digits still fit int8 lanes
    big = np.array([2 ** 31 - 1, -2 ** 31, 2 ** 30, -(2 ** 30) - 7], dtype=np.int64)
    b0, b1, b2 = digits3(big)
    assert np.array_equal(65536 * b0 + 256 * b1 + b2, big)


@pytest.mark.parametrize("scale", [1e-30, 1e-6, 1.0, 3.7e3, 6e6, 1e30])
def test_image_bounds(scale):
    rng = np.random.default_rng(1)
    v = (rng.standard_normal(2048) * scale).astype(np.float32)
    n, k = image(v)
    assert np.abs(n).max() <= 2 ** 22
    m = np.abs(v.astype(np.float64)).max()
    # the largest element keeps >= 21 bits: |n| >= 2^21 at the maximum
    assert np.abs(n).max() >= 2 ** 21
    # every element's rounding error is at most half a unit of the image
    err = np.abs(n * 2.0 ** -k - v.astype(np.float64))
    assert err.max() <= 0.5 * 2.0 ** -k and 2.0 ** -k <= m * 2.0 ** -21


def test_image_special_vectors():
    assert digit_shift(0) == 0                                   # all-zero vector: n = 0
    assert digit_shift(0x7F800000) == 0 and digit_shift(0x7FC00000) == 0   # inf / NaN: the kernel's NaN scale
    assert digit_shift(1) == 126                                 # subnormal max: clamped, |n| stays tiny
    n, k = image(np.full(64, 1e-45, np.float32))
    assert k == 126 and np.abs(n).max() <= 1


@pytest.mark.parametrize("seed,scale,outlier", [(0, 1.0, False), (1, 1e-3, True), (2, 2.5e3, False),
                                                (3, 6e6, True), (4, 0.05, True)])
def test_dot_matches_f64(seed, scale, outlier):
    rng = np.random.default_rng(seed)
    blocks = q4k.synth_blocks(seed, 77, 0, 8)          # one 2048-long gate/up row
    v = (rng.standard_normal(2048) * scale).astype(np.float32)
    if outlier:
        v[rng.integers(0, 2048)] = np.float32(40 * scale)
    w = q4k.dequant(blocks.tobytes()).astype(np.float64)
    exact = float(w @ v.astype(np.float64))
    got = digit_dot(blocks, v)
    m = float(np.abs(v.astype(np.float64)).max())
    bound = float(np.abs(w).sum()) * m * 2.0 ** -22   # rounding of v (half unit at 2^-21 m), doubled
    assert abs(got - exact) <= bound, (got, exact, bound)
    # relative to the dot's natural scale ||w|| ||v|| (Cauchy-Schwarz): ~1e-7 in practice
    rel = abs(got - exact) / (float(np.linalg.norm(w)) * float(np.linalg.norm(v.astype(np.float64))))
    assert rel < 2e-6, rel


def test_down_row_len_512():
    rng = np.random.default_rng(9)
    blocks = q4k.synth_blocks(3, 78, 0, 2)             # one 512-long down row
    s = (rng.standard_normal(512) * 3e3).astype(np.float32)
    w = q4k.dequant(blocks.tobytes()).astype(np.float64)
    exact = float(w @ s.astype(np.float64))
    got = digit_dot(blocks, s)
    assert abs(got - exact) <= float(np.abs(w).sum()) * float(np.abs(s).max()) * 2.0 ** -22
