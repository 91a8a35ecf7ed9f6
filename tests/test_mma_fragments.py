"""The fragment index algebra of the int8 tensor-core Q4_K dots (csrc/persist.cu q4k_mma_rows,
csrc/grouped.cu group_rows), checked exactly on the CPU.

The kernels assemble the operands of `mma.sync.m16n8k32.row.col.s32.s8.s8.s32` lane by lane:
lane = 4 g + t loads 8 consecutive quant bytes (8t..8t+7 of a 32-byte group) of two rows (MMA rows
g and g + 8); the low nibbles form the A registers of the group's first sub-block, the high
nibbles those of its second (a0 / a1 = bytes 0-3 of rows g / g + 8, a2 / a3 = bytes 4-7); B column
g holds digit plane g & 3 of token g >> 2 (plane 3 zero) at the same elements; D lands in lanes by
PTX's layout (c0, c1 = row g, columns 2t, 2t+1; c2, c3 = row g + 8). This model applies PTX's
fragment layout for m16n8k32 .s8 (A: row g for registers 0 and 2, g + 8 for 1 and 3, k = 4t + i,
+16 for registers 2 and 3; B: k = 4t + i, +16 for register 1, column g) and checks that every lane
then holds the exact integer sum(q * digit) of its rows, sub-block and column -- the identity the
kernels' scale and token bookkeeping rests on.
"""
import numpy as np


def _s8(x):
    x = np.asarray(x, dtype=np.int64) & 255
    return np.where(x >= 128, x - 256, x)


def mma_from_lanes(a_regs, b_regs):
    """a_regs [32, 4] u32, b_regs [32, 2] u32 (each 4 s8 bytes) -> per-lane c [32, 4] (PTX layout)."""
    A = np.zeros((16, 32), np.int64)
    B = np.zeros((32, 8), np.int64)
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        for r in range(4):
            row = g if r in (0, 2) else g + 8
            k0 = 4 * t + (16 if r >= 2 else 0)
            for i in range(4):
                A[row, k0 + i] = _s8(int(a_regs[lane, r]) >> (8 * i))
        for r in range(2):
            for i in range(4):
                B[4 * t + i + 16 * r, g] = _s8(int(b_regs[lane, r]) >> (8 * i))
    D = A @ B
    c = np.zeros((32, 4), np.int64)
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        c[lane] = [D[g, 2 * t], D[g, 2 * t + 1], D[g + 8, 2 * t], D[g + 8, 2 * t + 1]]
    return c


def _word(b4):
    return int(b4[0]) | int(b4[1]) << 8 | int(b4[2]) << 16 | int(b4[3]) << 24


def test_two_token_columns_give_exact_subblock_sums():
    rng = np.random.default_rng(0)
    qs = rng.integers(0, 256, (16, 32), dtype=np.int64)   # one 32-byte quant group of 16 rows
    # digit planes of two tokens over the group's 64 elements (low sub-block 0..31, high 32..63)
    dig = rng.integers(-128, 128, (2, 3, 64), dtype=np.int64)
    lo, hi = qs & 15, qs >> 4                              # the two sub-blocks' quants
    for half, q in ((0, lo), (1, hi)):
        a = np.zeros((32, 4), np.uint64)
        b = np.zeros((32, 2), np.uint64)
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            ra, rb = q[g, 8 * t:8 * t + 8], q[g + 8, 8 * t:8 * t + 8]
            a[lane] = [_word(ra[0:4]), _word(rb[0:4]), _word(ra[4:8]), _word(rb[4:8])]
            plane, tok = g & 3, g >> 2
            if plane < 3:
                d = dig[tok, plane, 32 * half + 8 * t:32 * half + 8 * t + 8]
                b[lane] = [_word(d[0:4] & 255), _word(d[4:8] & 255)]
        c = mma_from_lanes(a, b)
        want = q @ dig[:, :, 32 * half:32 * half + 32].reshape(6, 32).T   # [16 rows, token*3 + plane]
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            for j, (row, col) in enumerate(((g, 2 * t), (g, 2 * t + 1), (g + 8, 2 * t), (g + 8, 2 * t + 1))):
                tok, plane = col >> 2, col & 3          # column 4 tok + plane, plane 3 empty
                expect = 0 if plane == 3 else want[row, 3 * tok + plane]
                assert c[lane, j] == expect, (half, lane, j)


def test_lane_pairs_reduce_each_token_the_same_way():
    """Token A's planes sit in lanes t = 0, 1 and token B's in t = 2, 3 with the same column
    roles (plane 0 and 1 in the even lane, plane 2 in the odd one), so the kernels' per-lane
    weights (65536, 256 | 1, 0) and one xor-1 sum give both tokens the same operation sequence."""
    roles = {}
    for t in range(4):
        cols = (2 * t, 2 * t + 1)
        roles[t] = tuple((c >> 2, c & 3) for c in cols)
    assert [p for _, p in roles[0]] == [p for _, p in roles[2]] == [0, 1]
    assert [p for _, p in roles[1]] == [p for _, p in roles[3]] == [2, 3]
    assert {tk for tk, _ in roles[0] + roles[1]} == {0} and {tk for tk, _ in roles[2] + roles[3]} == {1}
