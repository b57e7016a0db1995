"""CPU check of the batch-1 K-quant GEMV's fragment mapping (csrc/rcu_gemv_kq.cu).

The kernel forms block dot products with mma.sync.m16n8k32 (u8 weights x s8 activations):
A holds 16 weight rows, B is block-diagonal (column j carries the activations of A's column
chunk j / 2), and each thread applies the scales of its own chunk's group. This test builds
every thread's registers exactly as the kernel does, multiplies them with the PTX ISA's
m16n8k32 8-bit fragment layouts, applies the per-thread scale / min arithmetic, and checks
that the pieces add up, per superblock and row, to the oracle's exact integer sums (sumi and
summ of quant/reference.rs:295-386). It also checks that the kernel's shared-memory loads are
aligned and free of bank conflicts for its padded row stride.
"""
import numpy as np
import pytest

import oracle as O

BB = {O.Q4_K: 144, O.Q5_K: 176, O.Q6_K: 210}
M4 = 0x0F0F0F0F


def word(buf, off):
    return int.from_bytes(bytes(buf[off:off + 4]), "little")


def sext8(x):
    x &= 0xFF
    return x - 256 if x >= 128 else x


def s16(x):
    x &= 0xFFFF
    return x - 65536 if x >= 32768 else x


def mma(a_regs, b_regs):
    """m16n8k32 .row.col s32 = u8 x s8 (+0): A / B / D fragments per lane, PTX ISA layouts."""
    A = np.zeros((16, 32), np.int64)
    B = np.zeros((32, 8), np.int64)
    for lane in range(32):
        g, c = lane >> 2, lane & 3
        for i in range(16):  # a0..a15 in 4 registers
            v = (a_regs[lane][i >> 2] >> (8 * (i & 3))) & 0xFF
            row = g if (i < 4 or 8 <= i < 12) else g + 8
            col = 4 * c + (i & 3) + (16 if i >= 8 else 0)
            A[row, col] = v
        for i in range(8):  # b0..b7 in 2 registers
            v = sext8(b_regs[lane][i >> 2] >> (8 * (i & 3)))
            B[4 * c + (i & 3) + (16 if i >= 4 else 0), g] = v
    D = A @ B
    return [(D[l >> 2, 2 * (l & 3)], D[l >> 2, 2 * (l & 3) + 1], D[(l >> 2) + 8, 2 * (l & 3)],
             D[(l >> 2) + 8, 2 * (l & 3) + 1]) for l in range(32)]


def pad_stride(row_bytes):
    return row_bytes + (16 + 128 - row_bytes % 128) % 128


def emulate(t, rows, act, nsb):
    """Per (row, superblock) integer sums formed by the kernel's threads: (sumi, summ)."""
    bb = BB[t]
    ps = pad_stride(nsb * bb)
    stage = np.zeros(16 * ps, np.uint8)
    for r in range(16):
        stage[r * ps:r * ps + nsb * bb] = rows[r]
    aq = act["qs"].reshape(-1).astype(np.int8).view(np.uint8)
    bsums = act["bsums"].reshape(-1).astype(np.int64)
    out = np.zeros((16, nsb, 2), np.int64)
    for sb in range(nsb):
        so = sb * bb
        lanes = [(l >> 2, l & 3) for l in range(32)]
        offs = [(g * ps, (g + 8) * ps) for g, c in lanes]
        bact = [c == (g >> 1) for g, c in lanes]
        if t in (O.Q4_K, O.Q5_K):
            qo = 16 if t == O.Q4_K else 48
            W = [[[word(stage, o + so + qo + 32 * c + 4 * i) for i in range(8)] for o in offs[l]]
                 for l, (g, c) in enumerate(lanes)]
            H = [[[word(stage, o + so + 16 + 4 * i) for i in range(8)] for o in offs[l]] for l in range(32)]
            AL = [[word(aq, sb * 256 + 64 * c + 4 * i) if bact[l] else 0 for i in range(8)]
                  for l, (g, c) in enumerate(lanes)]
            AH = [[word(aq, sb * 256 + 64 * c + 32 + 4 * i) if bact[l] else 0 for i in range(8)]
                  for l, (g, c) in enumerate(lanes)]

            def val(l, r, i, hi):
                c = lanes[l][1]
                w = W[l][r][i]
                if t == O.Q4_K:
                    return w & (0xF0F0F0F0 if hi else M4)
                h = H[l][r][i]
                if hi:
                    return ((w >> 4) & M4) | (((h >> (2 * c + 1)) & 0x01010101) << 4)
                return (w & M4) | (((h >> (2 * c)) & 0x01010101) << 4)
            DL = np.zeros((32, 4), np.int64)
            DH = np.zeros((32, 4), np.int64)
            for step in range(4):
                for hi, D, AX in ((0, DL, AL), (1, DH, AH)):
                    a = [(val(l, 0, 2 * step, hi), val(l, 1, 2 * step, hi), val(l, 0, 2 * step + 1, hi),
                          val(l, 1, 2 * step + 1, hi)) for l in range(32)]
                    b = [(AX[l][2 * step], AX[l][2 * step + 1]) for l in range(32)]
                    D += np.array(mma(a, b), np.int64)
            for l, (g, c) in enumerate(lanes):
                assert DL[l, 0] == DL[l, 1] and DH[l, 2] == DH[l, 3]  # duplicate columns 2c, 2c + 1
                for r, row in ((0, g), (1, g + 8)):
                    o = offs[l][r] + so
                    y, z, w_ = word(stage, o + 4), word(stage, o + 8), word(stage, o + 12)
                    sh = 16 * (c & 1)
                    a_, b_, cc = y >> sh, w_ >> sh, z >> sh
                    scp = a_ if c < 2 else (b_ & 0x0F0F) | ((a_ >> 2) & 0x3030)
                    mnp = cc if c < 2 else ((b_ >> 4) & 0x0F0F) | ((cc >> 2) & 0x3030)
                    dl, dh = int(DL[l, 2 * r]), int(DH[l, 2 * r])
                    if t == O.Q4_K:
                        assert dh % 16 == 0
                        dh >>= 4
                    I = (scp & 63) * dl + ((scp >> 8) & 63) * dh
                    bp_lo = bsums[16 * sb + 4 * c] + bsums[16 * sb + 4 * c + 1]
                    bp_hi = bsums[16 * sb + 4 * c + 2] + bsums[16 * sb + 4 * c + 3]
                    M = (mnp & 63) * bp_lo + ((mnp >> 8) & 63) * bp_hi
                    out[row, sb] += (I, M)
        else:  # Q6_K: thread c owns groups (n = c / 2, m = 0..3, h = c % 2); words rotated by c
            def ld(o, c):
                return [word(stage, o + 4 * ((i + c) & 3)) for i in range(4)]
            regs = []
            for l, (g, c) in enumerate(lanes):
                n, h = c >> 1, c & 1
                per = []
                for o in offs[l]:
                    per.append((ld(o + so + 64 * n + 16 * h, c), ld(o + so + 64 * n + 32 + 16 * h, c),
                                ld(o + so + 128 + 32 * n + 16 * h, c)))
                X = [[word(aq, sb * 256 + 128 * n + 32 * m + 16 * h + 4 * ((i + c) & 3)) if bact[l] else 0
                      for i in range(4)] for m in range(4)]
                regs.append((per, X))

            def q6(m, l0, l1, hh):
                if m == 0:
                    return (l0 & M4) | ((hh << 4) & 0x30303030)
                if m == 1:
                    return (l1 & M4) | ((hh << 2) & 0x30303030)
                if m == 2:
                    return ((l0 >> 4) & M4) | (hh & 0x30303030)
                return ((l1 >> 4) & M4) | ((hh >> 2) & 0x30303030)
            D = np.zeros((4, 32, 4), np.int64)
            for m in range(4):
                for u in range(2):
                    a, b = [], []
                    for l in range(32):
                        per, X = regs[l]
                        v = [q6(m, per[r][0][i], per[r][1][i], per[r][2][i]) & 0xFFFFFFFF
                             for r, i in ((0, 2 * u), (1, 2 * u), (0, 2 * u + 1), (1, 2 * u + 1))]
                        a.append(tuple(v))
                        b.append((X[m][2 * u], X[m][2 * u + 1]))
                    D[m] += np.array(mma(a, b), np.int64)
            for l, (g, c) in enumerate(lanes):
                n, h = c >> 1, c & 1
                for r, row in ((0, g), (1, g + 8)):
                    o = offs[l][r] + so
                    S = (word(stage, o + 192 + 8 * n), word(stage, o + 196 + 8 * n))
                    I = 0
                    for m in range(4):
                        sc = sext8(S[m >> 1] >> (8 * (h + 2 * (m & 1))))
                        I += sc * (int(D[m, l, 2 * r]) - 32 * int(bsums[16 * sb + 8 * n + 2 * m + h]))
                    out[row, sb, 0] += I
    return out


@pytest.mark.parametrize("t", [O.Q4_K, O.Q5_K, O.Q6_K], ids=["Q4_K", "Q5_K", "Q6_K"])
def test_fragment_sums_match_oracle(t):
    nsb = 3
    k = 256 * nsb
    rng = O.Rng(100 + t)
    w = rng.weight(t, 16, k)
    x = rng.vec(k, 1.0)
    act = O.quantize_row_q8_k(x)
    got = emulate(t, w, act, nsb)
    for r in range(16):
        ref = O.block_sums(t, w[r], act, k)
        if t == O.Q6_K:
            np.testing.assert_array_equal(got[r, :, 0], ref)
        else:
            np.testing.assert_array_equal(got[r].reshape(-1), ref)


def conflict_factor(addrs, width):
    """Shared-memory wavefronts of one warp-wide load over the ideal count (128 B each)."""
    per = 128 // width
    waves = 0
    for q in range(0, 32, per):
        banks = {}
        for a in addrs[q:q + per]:
            assert a % width == 0
            for w in range(width // 4):
                banks.setdefault((a // 4 + w) % 32, set()).add(a // 4 + w)
        waves += max(len(s) for s in banks.values())
    return waves / (32 * width // 128)


@pytest.mark.parametrize("t,k", [(O.Q4_K, 4096), (O.Q4_K, 2048), (O.Q5_K, 4096), (O.Q6_K, 4096),
                                 (O.Q6_K, 12288)])
def test_shared_loads_conflict_free(t, k):
    bb = BB[t]
    sl = 16 if k >= 4096 else 8
    ps = pad_stride(sl * bb)
    lanes = [(l >> 2, l & 3) for l in range(32)]
    for sbl in range(sl):
        so = sbl * bb
        if t != O.Q6_K:
            qo = 16 if t == O.Q4_K else 48
            for u in range(2):
                assert conflict_factor([g * ps + so + qo + 32 * c + 16 * u for g, c in lanes], 16) == 1
            assert conflict_factor([g * ps + so for g, c in lanes], 16) == 1
        else:
            for i in range(4):
                for base in (lambda n, h: 64 * n + 16 * h, lambda n, h: 64 * n + 32 + 16 * h,
                             lambda n, h: 128 + 32 * n + 16 * h):
                    ad = [(g * ps + so + base(c >> 1, c & 1) + 4 * ((i + c) & 3)) & ~3 for g, c in lanes]
                    assert conflict_factor(ad, 4) == 1
                    assert conflict_factor([a + 4 for a in ad], 4) == 1


def emulate_q4_0(rows, act_blocks, n_units):
    """Q4_0 units (8 blocks of 18 bytes) as k_gemv_kq forms them: per block one mma with A's
    chunk c = bytes 4c..4c+3 of the block (low nibbles at k 4c.., high at 16 + 4c..) and B the
    block's 32 codes in every column; thread c of each row group combines block 4 s + c of every
    four. Returns the per-(row, block) integer sums sum(nib * q) - 8 * sum(q) the threads form."""
    ps = pad_stride(n_units * 144)
    stage = np.zeros(16 * ps, np.uint8)
    for r in range(16):
        stage[r * ps:r * ps + n_units * 144] = rows[r]
    qs = act_blocks["qs"].astype(np.int8).view(np.uint8)  # [blocks][32]
    lanes = [(l >> 2, l & 3) for l in range(32)]
    out = np.zeros((16, 8 * n_units), np.int64)
    for u in range(n_units):
        so = u * 144
        for s4 in range(2):
            D = []
            for j in range(4):
                b = 4 * s4 + j
                blk = 8 * u + b
                a, bb = [], []
                for l, (g, c) in enumerate(lanes):
                    off = so + 18 * b + 2 + 4 * c
                    wa, wb = word(stage, g * ps + off), word(stage, (g + 8) * ps + off)
                    a.append((wa & M4, wb & M4, (wa >> 4) & M4, (wb >> 4) & M4))
                    bb.append((word(qs[blk], 4 * c), word(qs[blk], 16 + 4 * c)))
                D.append(mma(a, bb))
            for l, (g, c) in enumerate(lanes):
                blk = 8 * u + 4 * s4 + c
                sa = int(act_blocks["qs"][blk].astype(np.int64).sum())
                for r, row in ((0, g), (2, g + 8)):
                    out[row, blk] = int(D[c][l][r]) - 8 * sa
    return out


def test_q4_0_fragment_sums_match_oracle():
    n_units = 2
    k = 256 * n_units
    rng = O.Rng(404)
    w = rng.weight(O.Q4_0, 16, k)
    x = rng.vec(k, 1.0)
    act = O.quantize_row_q8_0(x, O.PATH_AVX2)
    got = emulate_q4_0(w, act, n_units)
    for r in range(16):
        np.testing.assert_array_equal(got[r], O.block_sums(O.Q4_0, w[r], act, k))


def test_q4_0_shared_loads_conflict_free():
    ps = pad_stride(16 * 144)
    lanes = [(l >> 2, l & 3) for l in range(32)]
    for b in range(8):
        ad = [(g * ps + 18 * b + 2 + 4 * c) & ~3 for g, c in lanes]
        assert conflict_factor(ad, 4) == 1
