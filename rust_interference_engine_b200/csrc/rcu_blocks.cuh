// rcu_blocks.cuh -- per-block integer dot products of GGUF weight blocks with int8
// activation codes, shared by the GEMV, the GEMM epilogue checks and rcu_block_sums.
//
// Each function returns the exact int32 the reference's scalar kernel forms for that
// block (crates/rie-core/src/quant/reference.rs:221-386); the f32 combine is done by the
// caller. `base` may point to shared or global memory; `off` is the block's byte offset
// and is only required to be even (GGUF blocks of 18/22/34/210 bytes are 2-aligned).
#pragma once
#include "rcu_internal.cuh"

namespace rcu {

// n consecutive 32-bit words starting at an even byte offset `off` from a 4-byte aligned
// base (the aligned words around the span are loaded and funnel-shifted into place).
template <int N>
__device__ __forceinline__ void ld_words(const uint8_t *base, uint64_t off, uint32_t (&out)[N]) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(base + (off & ~(uint64_t)3));
    const uint32_t sh = (uint32_t)(off & 3u) * 8u;
    uint32_t r[N + 1];
#pragma unroll
    for (int i = 0; i <= N; i++) r[i] = w[i];
#pragma unroll
    for (int i = 0; i < N; i++) out[i] = __funnelshift_rc(r[i], r[i + 1], sh);
}

// Spread 4 bits (h & 0xF) to bit 4 of each byte.
__device__ __forceinline__ uint32_t spread4_bit4(uint32_t h) { return (((h & 0xFu) * 0x00204081u) & 0x01010101u) << 4; }

// dp4a with unsigned weight bytes: codes 0..255 (e.g. a nibble in the high half of a byte,
// i.e. 16 x nibble) times signed activation bytes.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// Two int16 halves of a times the two low int8 bytes of b, plus c.
__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// Byte i (0..3) of w as a sign-extended int (i is a compile-time or lane constant).
__device__ __forceinline__ int sbyte(uint32_t w, uint32_t i) { return (int)(int8_t)((w >> (8 * i)) & 0xffu); }

// ---- 32-value blocks (activations: 32 int8 codes as 8 words, their exact sum) --------
// A block at an even byte offset is read as the aligned words around it; one funnel shift
// per word (by 16 or by 32, i.e. none) puts each field in place.
struct BlkW {  // decoded weight block
    uint32_t v[8];  // Q4: v[0..3] low nibbles, v[4..7] = 16 x high nibbles; Q5/Q8: codes
    float d, m;     // f16 scale (and min for Q4_1/Q5_1) as f32
};

// Q4_0 (reference.rs:55-62, :221-233): codes nib-8; we keep nib and subtract 8*sum(a).
__device__ __forceinline__ void dec_q4_0(const uint8_t *b, uint32_t off, BlkW &o) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(b + (off & ~3u));
    const uint32_t sh = (off & 3u) * 8u;  // 0 or 16
    uint32_t r[5];
#pragma unroll
    for (int i = 0; i < 5; i++) r[i] = w[i];
    o.d = f16_bits_to_f32(__funnelshift_rc(r[0], r[1], sh));
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t q = __funnelshift_rc(r[i], r[i + 1], sh + 16);
        o.v[i] = q & 0x0F0F0F0Fu;
        o.v[4 + i] = q & 0xF0F0F0F0u;
    }
    o.m = 0.0f;
}
// Q4_1 (reference.rs:63-71, :235-247): 20-byte blocks are 4-aligned.
__device__ __forceinline__ void dec_q4_1(const uint8_t *b, uint32_t off, BlkW &o) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(b + off);
    const uint32_t h = w[0];
    o.d = f16_bits_to_f32(h);
    o.m = f16_bits_to_f32(h >> 16);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t q = w[1 + i];
        o.v[i] = q & 0x0F0F0F0Fu;
        o.v[4 + i] = q & 0xF0F0F0F0u;
    }
}
// Q5_0 (reference.rs:72-82, :249-264): 5th bit j of qh -> element j, bit j+16 -> j+16.
__device__ __forceinline__ void dec_q5_0(const uint8_t *b, uint32_t off, BlkW &o) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(b + (off & ~3u));
    const uint32_t sh = (off & 3u) * 8u;
    uint32_t r[6];
#pragma unroll
    for (int i = 0; i < 6; i++) r[i] = w[i];
    o.d = f16_bits_to_f32(__funnelshift_rc(r[0], r[1], sh));
    const uint32_t qh = __funnelshift_rc(r[0], r[1], sh + 16);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t q = __funnelshift_rc(r[1 + i], r[2 + i], sh + 16);
        o.v[i] = (q & 0x0F0F0F0Fu) | spread4_bit4(qh >> (4 * i));
        o.v[4 + i] = ((q >> 4) & 0x0F0F0F0Fu) | spread4_bit4(qh >> (16 + 4 * i));
    }
    o.m = 0.0f;
}
// Q5_1 (reference.rs:83-94, :266-281): 24-byte blocks are 8-aligned.
__device__ __forceinline__ void dec_q5_1(const uint8_t *b, uint32_t off, BlkW &o) {
    const uint2 *w = reinterpret_cast<const uint2 *>(b + off);
    const uint2 h = w[0], q01 = w[1], q23 = w[2];
    o.d = f16_bits_to_f32(h.x);
    o.m = f16_bits_to_f32(h.x >> 16);
    const uint32_t qh = h.y, qw[4] = {q01.x, q01.y, q23.x, q23.y};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        o.v[i] = (qw[i] & 0x0F0F0F0Fu) | spread4_bit4(qh >> (4 * i));
        o.v[4 + i] = ((qw[i] >> 4) & 0x0F0F0F0Fu) | spread4_bit4(qh >> (16 + 4 * i));
    }
}
// Q8_0 (reference.rs:95-100, :283-293)
__device__ __forceinline__ void dec_q8_0(const uint8_t *b, uint64_t off, BlkW &o) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(b + (off & ~(uint64_t)3));
    const uint32_t sh = (uint32_t)(off & 3u) * 8u;
    uint32_t r[9];
#pragma unroll
    for (int i = 0; i < 9; i++) r[i] = w[i];
    o.d = f16_bits_to_f32(__funnelshift_rc(r[0], r[1], sh));
#pragma unroll
    for (int i = 0; i < 8; i++) o.v[i] = __funnelshift_rc(r[i], r[i + 1], sh + 16);
    o.m = 0.0f;
}

template <int TYPE>
__device__ __forceinline__ void dec_blk(const uint8_t *b, uint32_t off, BlkW &o) {
    if (TYPE == T_Q4_0) dec_q4_0(b, off, o);
    if (TYPE == T_Q4_1) dec_q4_1(b, off, o);
    if (TYPE == T_Q5_0) dec_q5_0(b, off, o);
    if (TYPE == T_Q5_1) dec_q5_1(b, off, o);
    if (TYPE == T_Q8_0) dec_q8_0(b, off, o);
}
// Exact integer block sum s of the reference (offset-coded types subtract 8 / 16 x sum(a)).
template <int TYPE>
__device__ __forceinline__ int blk_int(const BlkW &w, const uint32_t (&a)[8], int asum) {
    if (TYPE == T_Q4_0 || TYPE == T_Q4_1) {
        int lo = 0, hi = 0;  // hi accumulates 16 x (high nibble . a)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            lo = dp4a_us(w.v[i], a[i], lo);
            hi = dp4a_us(w.v[4 + i], a[4 + i], hi);
        }
        const int s = lo + (hi >> 4);
        return TYPE == T_Q4_0 ? s - 8 * asum : s;
    }
    int s0 = 0, s1 = 0;  // two chains halve the dp4a dependency latency
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        s0 = dp4a(w.v[i], a[i], s0);
        s1 = dp4a(w.v[i + 1], a[i + 1], s1);
    }
    int s = s0 + s1;
    if (TYPE == T_Q5_0) s -= 16 * asum;
    return s;
}
template <int TYPE>
constexpr int blk_bytes_c() {
    return TYPE == T_Q4_0 ? 18 : TYPE == T_Q4_1 ? 20 : TYPE == T_Q5_0 ? 22 : TYPE == T_Q5_1 ? 24 : 34;
}

// get_scale_min_k4 (reference.rs:8-14) on the 12 scale bytes held in 3 words (dequantize path).
__device__ __forceinline__ void scale_min_k4(int j, const uint32_t (&s)[3], uint32_t &sc, uint32_t &mn) {
    auto byte = [&](int i) -> uint32_t { return (s[i >> 2] >> (8 * (i & 3))) & 0xffu; };
    if (j < 4) {
        sc = byte(j) & 63u;
        mn = byte(j + 4) & 63u;
    } else {
        sc = (byte(j + 4) & 0xFu) | ((byte(j - 4) >> 6) << 4);
        mn = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}

// ---- 256-value superblocks, 8 cooperating lanes per superblock ----------------------
// Q4_K / Q5_K: lane `sub` (0..7) owns elements [64j + 16h, +16) (sub-block 2j) and
// [64j + 32 + 16h, +16) (sub-block 2j+1) with j = sub/2, h = sub%2, and the min of
// sub-block `sub` (whose 32 activations are Q8_K bsums 2*sub and 2*sub+1). The lane's share
// of the superblock's exact sums is
//   I = sc[2j] * (w_lo . a_lo) + sc[2j+1] * (w_hi . a_hi),  M = mn[sub] * (bsums pair)
// and the eight lanes' shares add up to the reference's sumi / summ (reference.rs:295-350).
struct KLane {  // lane constants
    uint32_t sub, j, h, sh16, csh;
    bool hi;
};
__device__ __forceinline__ KLane k_lane(uint32_t sub) {
    KLane l;
    l.sub = sub;
    l.j = sub >> 1;
    l.h = sub & 1;
    l.sh16 = 16 * (l.j & 1);
    l.csh = 8 * (sub & 3);
    l.hi = sub >= 4;
    return l;
}
// Scales sc[2j], sc[2j+1] and min mn[sub] from the 12 scale bytes s0..s2
// (get_scale_min_k4, reference.rs:8-14).
__device__ __forceinline__ void k_scales(const KLane &l, uint32_t s0, uint32_t s1, uint32_t s2, int &sc_lo, int &sc_hi,
                                         int &mn) {
    const uint32_t a = s0 >> l.sh16, b = s2 >> l.sh16;
    const uint32_t pair = l.hi ? ((b & 0x0F0Fu) | ((a >> 2) & 0x3030u)) : a;
    sc_lo = (int)(pair & 63u);
    sc_hi = (int)((pair >> 8) & 63u);
    const uint32_t c = s1 >> l.csh, d = s2 >> l.csh;
    const uint32_t m = l.hi ? (((d >> 4) & 0x0Fu) | ((c >> 2) & 0x30u)) : c;
    mn = (int)(m & 63u);
}
// Lane share (I, M) of one Q4_K (144 B) or Q5_K (176 B) superblock at 16-aligned `sb`;
// alo / ahi: the lane's 16 + 16 activation codes, bs2: bsums[2*sub] | bsums[2*sub+1] << 16.
// Returns the packed f16 pair (d, dmin).
template <int TYPE>
__device__ __forceinline__ uint32_t k_lane_dot(const KLane &l, const uint8_t *sb, const uint4 &alo, const uint4 &ahi,
                                               uint32_t bs2, int &I, int &M) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(sb);
    int sc_lo, sc_hi, mn;
    k_scales(l, hdr.y, hdr.z, hdr.w, sc_lo, sc_hi, mn);
    const uint32_t al[4] = {alo.x, alo.y, alo.z, alo.w}, ah[4] = {ahi.x, ahi.y, ahi.z, ahi.w};
    int s1 = 0, s2 = 0;
    if (TYPE == T_Q4_K) {
        const uint4 q = *reinterpret_cast<const uint4 *>(sb + 16 + 32 * l.j + 16 * l.h);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            s1 = dp4a_us(qw[i] & 0x0F0F0F0Fu, al[i], s1);
            s2 = dp4a_us(qw[i] & 0xF0F0F0F0u, ah[i], s2);
        }
        s2 >>= 4;  // exact: every term was 16 x nibble x a
    } else {  // qh[32] at 16, ql[128] at 48
        const uint4 qh = *reinterpret_cast<const uint4 *>(sb + 16 + 16 * l.h);
        const uint4 q = *reinterpret_cast<const uint4 *>(sb + 48 + 32 * l.j + 16 * l.h);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w}, hw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t lo = (qw[i] & 0x0F0F0F0Fu) | (((hw[i] >> (2 * l.j)) & 0x01010101u) << 4);
            const uint32_t hi = ((qw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * l.j + 1)) & 0x01010101u) << 4);
            s1 = dp4a_us(lo, al[i], s1);
            s2 = dp4a_us(hi, ah[i], s2);
        }
    }
    I = s1 * sc_lo + s2 * sc_hi;
    M = dp2a_lo(bs2, (uint32_t)mn * 0x0101u, 0);
    return hdr.x;
}

// Q6_K (reference.rs:190-207, :352-386). Lane `sub`: half n = sub/4, positions l in
// [8*lq, 8*lq+8) with lq = sub%4, covering elements 128n + 32k + l (k = 0..3). Exact:
//   sumi = sum_e sc[e/16] * q6[e] * a[e] - 32 * sum_g sc[g] * bsums[g]
// the lane's share of the second sum is its groups 2*sub, 2*sub+1 (one dp2a).
struct Q6Lane {
    uint32_t n, lq, is, sub;
};
__device__ __forceinline__ Q6Lane q6_lane(uint32_t sub) { return Q6Lane{sub >> 2, sub & 3, (sub & 3) >> 1, sub}; }
// Superblock at an even offset `off` from a 4-aligned base; a[k]: the lane's 8 activation
// codes of group k; bs2 = bsums[2*sub] | bsums[2*sub+1] << 16. Returns the f16 d bits.
__device__ __forceinline__ uint32_t q6_lane_dot(const Q6Lane &l, const uint8_t *base, uint32_t off, const uint2 (&a)[4],
                                                uint32_t bs2, int &I) {
    uint32_t A[2], B[2], H[2], S[2];
    ld_words<2>(base, off + 64 * l.n + 8 * l.lq, A);
    ld_words<2>(base, off + 64 * l.n + 32 + 8 * l.lq, B);
    ld_words<2>(base, off + 128 + 32 * l.n + 8 * l.lq, H);
    ld_words<2>(base, off + 192 + 8 * l.n, S);
    const uint32_t scp = *reinterpret_cast<const uint16_t *>(base + off + 192 + 2 * l.sub);
    const uint32_t dbits = *reinterpret_cast<const uint16_t *>(base + off + 208);
    int acc = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        int s = 0;
#pragma unroll
        for (int w = 0; w < 2; w++) {
            const uint32_t src = (k & 1) ? B[w] : A[w];
            const uint32_t lo4 = (k < 2) ? (src & 0x0F0F0F0Fu) : ((src >> 4) & 0x0F0F0F0Fu);
            const uint32_t q = lo4 | (((H[w] >> (2 * k)) & 0x03030303u) << 4);
            s = dp4a_us(q, w ? a[k].y : a[k].x, s);
        }
        const uint32_t sci = l.is + 2 * k;  // scale byte within this half: 0..7
        acc += sbyte(S[sci >> 2], sci & 3) * s;
    }
    I = acc - 32 * dp2a_lo(bs2, scp, 0);
    return dbits;
}

}  // namespace rcu
