"""CPU check of the turbo4 decode attention's tensor-core fragments (k_attn_dec_t4, csrc/rcu_attn_dec.cu).

The kernel scores 16 cache rows at a time with mma.m16n8k32 (level magnitudes x query codes) and
sums V with mma.m16n8k16 (f16 levels x f16 softmax weights). This test builds every lane's
registers as the kernel does -- the byte-permute lookups with their sign-replicating selectors,
the query codes in the A fragments' k order, the movmatrix transpose of the weights, the
dim-slot mapping of the V tiles -- multiplies them with the PTX ISA fragment layouts, and checks
  * that every (row, head, 32-dim block) score sum is the reference's exact int32 sum
    sum(level_i8[code] * q_i8) (turbo.rs:197-222);
  * that the V tiles hold sum_rows level_i8[code] * weight * 2^-24 for every dim and head, with the
    weights as the f16 sum hi + lo the kernel forms (turbo.rs:224-251 up to that rounding);
  * that every shared-memory load of a row lands on a 2-byte boundary.
The emulated prmt follows the PTX ISA's default mode: the three low bits of a selector nibble
pick one of the 8 source bytes, its high bit replicates that byte's sign bit instead.
"""
import numpy as np
import pytest

import oracle as O

LEVELS = np.array([-126, -95, -74, -58, -43, -30, -18, -6, 6, 18, 30, 43, 58, 74, 95, 126], np.int64)
T4_POS = (0x2b1e1206, 0x7e5f4a3a)
T4_NEG = (0x3a4a5f7e, 0x06121e2b)
RB = 66  # turbo4 row at head_dim 128: f16 scale, 64 code bytes


def prmt(a, b, c):
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    out = 0
    for i in range(4):
        n = (c >> (4 * i)) & 0xF
        v = src[n & 7]
        if n & 8:
            v = 0xFF if v & 0x80 else 0x00
        out |= v << (8 * i)
    return out


def t4_pos(sel):
    return prmt(T4_POS[0], T4_POS[1], sel)


def t4_neg(sel):
    return prmt(T4_NEG[0], T4_NEG[1], sel)


def sext8(x):
    x &= 0xFF
    return x - 256 if x >= 128 else x


def lds16(buf, off):
    assert off % 2 == 0, "unaligned 16-bit shared load"
    return int(buf[off]) | int(buf[off + 1]) << 8


def mma_k32(a_regs, b_regs):
    """m16n8k32 .row.col s32 = u8 x s8: per-lane D fragments (PTX ISA 8-bit layouts)."""
    A = np.zeros((16, 32), np.int64)
    B = np.zeros((32, 8), np.int64)
    for lane in range(32):
        g, c = lane >> 2, lane & 3
        for i in range(16):
            v = (a_regs[lane][i >> 2] >> (8 * (i & 3))) & 0xFF
            row = g if (i < 4 or 8 <= i < 12) else g + 8
            A[row, 4 * c + (i & 3) + (16 if i >= 8 else 0)] = v
        for i in range(8):
            B[4 * c + (i & 3) + (16 if i >= 4 else 0), g] = sext8(b_regs[lane][i >> 2] >> (8 * (i & 3)))
    D = A @ B
    return np.array([(D[l >> 2, 2 * (l & 3)], D[l >> 2, 2 * (l & 3) + 1], D[(l >> 2) + 8, 2 * (l & 3)],
                      D[(l >> 2) + 8, 2 * (l & 3) + 1]) for l in range(32)], np.int64)


def halves(x):
    return np.array([x & 0xFFFF, x >> 16], np.uint16).view(np.float16).astype(np.float64)


def mma_k16(a_regs, b_regs):
    """m16n8k16 .row.col f32 = f16 x f16, products summed exactly (f64 here)."""
    A = np.zeros((16, 16))
    B = np.zeros((16, 8))
    for lane in range(32):
        g, c = lane >> 2, lane & 3
        for r, (row, col) in enumerate(((g, 2 * c), (g + 8, 2 * c), (g, 2 * c + 8), (g + 8, 2 * c + 8))):
            A[row, col:col + 2] = halves(a_regs[lane][r])
        for r, k in enumerate((2 * c, 2 * c + 8)):
            B[k:k + 2, g] = halves(b_regs[lane][r])
    D = A @ B
    return np.array([(D[l >> 2, 2 * (l & 3)], D[l >> 2, 2 * (l & 3) + 1], D[(l >> 2) + 8, 2 * (l & 3)],
                      D[(l >> 2) + 8, 2 * (l & 3) + 1]) for l in range(32)])


def movmatrix_t(regs):
    """movmatrix.m8n8.trans.b16: lane (g, c) holds row g, columns 2c, 2c + 1 before and after."""
    M = np.zeros((8, 8), np.uint32)
    for lane in range(32):
        g, c = lane >> 2, lane & 3
        M[g, 2 * c], M[g, 2 * c + 1] = regs[lane] & 0xFFFF, regs[lane] >> 16
    T = M.T
    return [int(T[l >> 2, 2 * (l & 3)]) | int(T[l >> 2, 2 * (l & 3) + 1]) << 16 for l in range(32)]


def f16_bits(x):
    return int(np.float16(x).view(np.uint16))


def pack_s8(*v):
    return sum((int(x) & 0xFF) << (8 * i) for i, x in enumerate(v))


def codes_of(row_bytes):
    """Codes of a turbo4 row by dim (row_bytes_4 layout: chunk of 16 bytes per 32 dims)."""
    cb = row_bytes[2:]
    out = np.zeros(128, np.int64)
    for d in range(128):
        b = cb[16 * (d // 32) + d % 16]
        out[d] = (b >> 4) if (d % 32) >= 16 else (b & 15)
    return out


def make_stage(rng, n_rows, base):
    """A stage buffer holding n_rows turbo4 rows from an even byte offset."""
    buf = np.zeros(base + 16 * RB + 64, np.uint8)
    rows = rng.integers(0, 256, (16, RB), dtype=np.uint8)
    rows[:, 0:2] = np.frombuffer(np.float16(rng.uniform(0.01, 3.0, 16)).tobytes(), np.uint8).reshape(16, 2)
    for r in range(16):
        buf[base + r * RB:base + (r + 1) * RB] = rows[r]
    return buf, rows


@pytest.mark.parametrize("G", [8, 4])
@pytest.mark.parametrize("base", [0, 2, 14])
def test_score_block_sums_exact(G, base):
    rng = np.random.default_rng(G * 10 + base)
    buf, rows = make_stage(rng, 16, base)
    q = rng.integers(-127, 128, (G, 128))
    bq, bn = [], []
    for lane in range(32):
        g, c = lane >> 2, lane & 3
        lb, ln = [], []
        for ch in range(4):
            if g < G:
                qh = q[g, 32 * ch + 4 * c:]
                lb.append((pack_s8(qh[0], qh[16], qh[1], qh[17]), pack_s8(qh[2], qh[18], qh[3], qh[19])))
                ln.append((pack_s8(-qh[0], -qh[16], -qh[1], -qh[17]), pack_s8(-qh[2], -qh[18], -qh[3], -qh[19])))
            else:
                lb.append((0, 0))
                ln.append((0, 0))
        bq.append(lb)
        bn.append(ln)
    codes = np.stack([codes_of(rows[r]) for r in range(16)])
    for ch in range(4):
        ap, an = [], []
        for lane in range(32):
            g, c = lane >> 2, lane & 3
            og, og8 = base + g * RB, base + (g + 8) * RB
            wa = lds16(buf, og + 2 + 16 * ch + 4 * c) | lds16(buf, og + 2 + 16 * ch + 4 * c + 2) << 16
            wb = lds16(buf, og8 + 2 + 16 * ch + 4 * c) | lds16(buf, og8 + 2 + 16 * ch + 4 * c + 2) << 16
            xa, xb = wa ^ 0x88888888, wb ^ 0x88888888
            ap.append((t4_pos(xa), t4_pos(xb), t4_pos(xa >> 16), t4_pos(xb >> 16)))
            an.append((t4_neg(wa), t4_neg(wb), t4_neg(wa >> 16), t4_neg(wb >> 16)))
        D = mma_k32(ap, [bq[l][ch] for l in range(32)]) + mma_k32(an, [bn[l][ch] for l in range(32)])
        blk = slice(32 * ch, 32 * ch + 32)
        want = LEVELS[codes[:, blk]] @ q[:, blk].T  # [row, head]
        for lane in range(32):
            g, c = lane >> 2, lane & 3
            for i, (r, h) in enumerate(((g, 2 * c), (g, 2 * c + 1), (g + 8, 2 * c), (g + 8, 2 * c + 1))):
                if h < G:
                    assert D[lane, i] == want[r, h], (ch, lane, i)


@pytest.mark.parametrize("hilo", [True, False])
@pytest.mark.parametrize("base", [0, 6])
def test_v_tiles(hilo, base):
    G = 8
    rng = np.random.default_rng(7 + base)
    buf, rows = make_stage(rng, 16, base)
    W = rng.uniform(0.0, 1.0, (16, G)) ** 4  # weights in (0, 1], many small
    W[3, :] = 0.0
    W[:, 5] *= 1e-3
    W = W.astype(np.float32)
    Wh = W.astype(np.float16).astype(np.float32)
    Wl = (W - Wh).astype(np.float16).astype(np.float32)
    Weff = Wh.astype(np.float64) + (Wl.astype(np.float64) if hilo else 0.0)
    # weights in the scores' fragment layout (rows g, g + 8 x heads 2c, 2c + 1), then transposed
    hg = [f16_bits(W[l >> 2, 2 * (l & 3)]) | f16_bits(W[l >> 2, 2 * (l & 3) + 1]) << 16 for l in range(32)]
    hg8 = [f16_bits(W[(l >> 2) + 8, 2 * (l & 3)]) | f16_bits(W[(l >> 2) + 8, 2 * (l & 3) + 1]) << 16 for l in range(32)]
    lg = [f16_bits(W[l >> 2, 2 * (l & 3)] - Wh[l >> 2, 2 * (l & 3)]) |
          f16_bits(W[l >> 2, 2 * (l & 3) + 1] - Wh[l >> 2, 2 * (l & 3) + 1]) << 16 for l in range(32)]
    lg8 = [f16_bits(W[(l >> 2) + 8, 2 * (l & 3)] - Wh[(l >> 2) + 8, 2 * (l & 3)]) |
           f16_bits(W[(l >> 2) + 8, 2 * (l & 3) + 1] - Wh[(l >> 2) + 8, 2 * (l & 3) + 1]) << 16 for l in range(32)]
    bh = list(zip(movmatrix_t(hg), movmatrix_t(hg8)))
    bl = list(zip(movmatrix_t(lg), movmatrix_t(lg8)))
    nh = [(a ^ 0x80008000, b ^ 0x80008000) for a, b in bh]
    nl = [(a ^ 0x80008000, b ^ 0x80008000) for a, b in bl]
    O_ = np.zeros((8, 32, 4))
    for k in range(4):
        for e in range(2):
            P, N = [], []
            for lane in range(32):
                g, c = lane >> 2, lane & 3
                va, vb, vc, vd = (base + r * RB + 2 + 8 * g for r in (2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9))
                xab = prmt(lds16(buf, va + 2 * k), lds16(buf, vb + 2 * k), 0x5140)
                xcd = prmt(lds16(buf, vc + 2 * k), lds16(buf, vd + 2 * k), 0x5140)
                yab, ycd = xab ^ 0x88888888, xcd ^ 0x88888888
                pab, pcd = t4_pos(yab >> (16 * e)), t4_pos(ycd >> (16 * e))
                nab, ncd = t4_neg(xab >> (16 * e)), t4_neg(xcd >> (16 * e))
                P.append((prmt(pab, 0, 0x4240), prmt(pab, 0, 0x4341), prmt(pcd, 0, 0x4240), prmt(pcd, 0, 0x4341)))
                N.append((prmt(nab, 0, 0x4240), prmt(nab, 0, 0x4341), prmt(ncd, 0, 0x4240), prmt(ncd, 0, 0x4341)))
            t = 2 * k + e
            O_[t] += mma_k16(P, bh) + mma_k16(N, nh)
            if hilo:
                O_[t] += mma_k16(P, bl) + mma_k16(N, nl)
    codes = np.stack([codes_of(rows[r]) for r in range(16)])
    want = (LEVELS[codes].T.astype(np.float64) @ Weff) * 2.0 ** -24  # [dim, head]
    for lane in range(32):
        g, c = lane >> 2, lane & 3
        for t in range(8):
            d = 32 * (g >> 1) + 8 * (g & 1) + t
            got = O_[t, lane]
            np.testing.assert_allclose(got, [want[d, 2 * c], want[d, 2 * c + 1], want[d + 16, 2 * c],
                                             want[d + 16, 2 * c + 1]], rtol=1e-12, atol=1e-20)


def test_dim_slots_cover_every_dim_once():
    seen = set()
    for g in range(8):
        for t in range(8):
            d = 32 * (g >> 1) + 8 * (g & 1) + t
            seen.update((d, d + 16))
    assert seen == set(range(128))


def test_tables_are_the_level_magnitudes():
    for c in range(16):
        sel = c | 0x8880  # code in nibble 0; other nibbles read byte 0 sign-replicated (0)
        pos, neg = t4_pos(sel ^ 0x8), t4_neg(sel) & 0xFF
        assert (pos & 0xFF) - neg == LEVELS[c]
        assert pos >> 8 == 0
    assert O.turbo_quantize_4 is not None  # the oracle's codes use the same level order
