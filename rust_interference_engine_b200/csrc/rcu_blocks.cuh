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

// ---- 32-value blocks (activations: 32 int8 codes as 8 words, their exact sum) --------
struct BlkW {  // decoded weight block: 8 words of unsigned/signed codes in element order
    uint32_t v[8];
    float d, m;  // f16 scale (and min for Q4_1/Q5_1) as f32
};

// Q4_0 (reference.rs:55-62, :221-233): codes nib-8, we keep nib and subtract 8*sum(a).
__device__ __forceinline__ void dec_q4_0(const uint8_t *b, uint32_t off, BlkW &o) {
    uint32_t w[5];
    ld_words<5>(b, off, w);  // bytes off .. off+20
    o.d = f16_bits_to_f32(w[0]);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t q = __funnelshift_r(w[i], w[i + 1], 16);
        o.v[i] = q & 0x0F0F0F0Fu;
        o.v[4 + i] = (q >> 4) & 0x0F0F0F0Fu;
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
        o.v[4 + i] = (q >> 4) & 0x0F0F0F0Fu;
    }
}
// Q5_0 (reference.rs:72-82, :249-264): 5th bit j of qh -> element j, bit j+16 -> j+16.
__device__ __forceinline__ void dec_q5_0(const uint8_t *b, uint32_t off, BlkW &o) {
    uint32_t w[6];
    ld_words<6>(b, off, w);  // d(2) qh(4) qs(16)
    o.d = f16_bits_to_f32(w[0]);
    const uint32_t qh = __funnelshift_r(w[0], w[1], 16);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t q = __funnelshift_r(w[1 + i], w[2 + i], 16);
        o.v[i] = (q & 0x0F0F0F0Fu) | spread4_bit4(qh >> (4 * i));
        o.v[4 + i] = ((q >> 4) & 0x0F0F0F0Fu) | spread4_bit4(qh >> (16 + 4 * i));
    }
    o.m = 0.0f;
}
// Q5_1 (reference.rs:83-94, :266-281): 24-byte blocks are 4-aligned.
__device__ __forceinline__ void dec_q5_1(const uint8_t *b, uint32_t off, BlkW &o) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(b + off);
    o.d = f16_bits_to_f32(w[0]);
    o.m = f16_bits_to_f32(w[0] >> 16);
    const uint32_t qh = w[1];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t q = w[2 + i];
        o.v[i] = (q & 0x0F0F0F0Fu) | spread4_bit4(qh >> (4 * i));
        o.v[4 + i] = ((q >> 4) & 0x0F0F0F0Fu) | spread4_bit4(qh >> (16 + 4 * i));
    }
}
// Q8_0 (reference.rs:95-100, :283-293)
__device__ __forceinline__ void dec_q8_0(const uint8_t *b, uint64_t off, BlkW &o) {
    uint32_t w[9];
    ld_words<9>(b, off, w);
    o.d = f16_bits_to_f32(w[0]);
#pragma unroll
    for (int i = 0; i < 8; i++) o.v[i] = __funnelshift_r(w[i], w[i + 1], 16);
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
    int s0 = 0, s1 = 0;  // two chains halve the dp4a dependency latency
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        s0 = dp4a(w.v[i], a[i], s0);
        s1 = dp4a(w.v[i + 1], a[i + 1], s1);
    }
    int s = s0 + s1;
    if (TYPE == T_Q4_0) s -= 8 * asum;
    if (TYPE == T_Q5_0) s -= 16 * asum;
    return s;
}
template <int TYPE>
constexpr int blk_bytes_c() {
    return TYPE == T_Q4_0 ? 18 : TYPE == T_Q4_1 ? 20 : TYPE == T_Q5_0 ? 22 : TYPE == T_Q5_1 ? 24 : 34;
}

// ---- 256-value superblocks, 8 cooperating lanes per superblock ----------------------
// Lane `sub` (0..7) of the group owns elements [64j + 16h, +16) and [64j + 32 + 16h, +16)
// with j = sub/2, h = sub%2 (Q4_K/Q5_K), and the scale/min index `sub` for the min term.

// get_scale_min_k4 (reference.rs:8-14) on the 12 scale bytes held in 3 words.
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

struct SbAct {  // one lane's share of a Q8_K activation superblock
    uint4 lo, hi;  // 16 codes for the low-nibble and high-nibble sub-blocks
    uint32_t bs2;  // bsums[2*sub] | bsums[2*sub+1] << 16 (i16 pair)
    float d;
};
struct SbW {  // one lane's share of a decoded Q4_K / Q5_K weight superblock
    uint32_t lo[4], hi[4];
    int sc_lo, sc_hi, mn;
    float d, dmin;
};

// Q4_K (reference.rs:153-168) and Q5_K (reference.rs:169-189) decode of lane `sub`.
template <int TYPE>
__device__ __forceinline__ void dec_sb_k(const uint8_t *base, uint32_t off, int sub, SbW &o) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(base + off);
    o.d = f16_bits_to_f32(hdr.x);
    o.dmin = f16_bits_to_f32(hdr.x >> 16);
    const uint32_t s[3] = {hdr.y, hdr.z, hdr.w};
    const int j = sub >> 1, h = sub & 1;
    uint32_t a, b, c, m;
    scale_min_k4(2 * j, s, a, m);
    scale_min_k4(2 * j + 1, s, b, m);
    scale_min_k4(sub, s, c, m);
    o.sc_lo = (int)a;
    o.sc_hi = (int)b;
    o.mn = (int)m;
    uint4 q, qh = make_uint4(0, 0, 0, 0);
    if (TYPE == T_Q4_K) {
        q = *reinterpret_cast<const uint4 *>(base + off + 16 + 32 * j + 16 * h);
    } else {  // qh[32] at 16, ql[128] at 48
        qh = *reinterpret_cast<const uint4 *>(base + off + 16 + 16 * h);
        q = *reinterpret_cast<const uint4 *>(base + off + 48 + 32 * j + 16 * h);
    }
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        o.lo[i] = qw[i] & 0x0F0F0F0Fu;
        o.hi[i] = (qw[i] >> 4) & 0x0F0F0F0Fu;
        if (TYPE == T_Q5_K) {
            o.lo[i] |= ((hw[i] >> (2 * j)) & 0x01010101u) << 4;
            o.hi[i] |= ((hw[i] >> (2 * j + 1)) & 0x01010101u) << 4;
        }
    }
}
// Lane share of sumi (sum_j s1*sc[2j] + s2*sc[2j+1]) and summ ((bsum pair) * mn[sub]).
__device__ __forceinline__ int dot_sb_k(const SbW &w, const SbAct &a, int &summ) {
    const uint32_t alo[4] = {a.lo.x, a.lo.y, a.lo.z, a.lo.w};
    const uint32_t ahi[4] = {a.hi.x, a.hi.y, a.hi.z, a.hi.w};
    int s1 = 0, s2 = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        s1 = dp4a(w.lo[i], alo[i], s1);
        s2 = dp4a(w.hi[i], ahi[i], s2);
    }
    const int bsum = (int)(int16_t)(a.bs2 & 0xffffu) + (int)(int16_t)(a.bs2 >> 16);
    summ = bsum * w.mn;
    return s1 * w.sc_lo + s2 * w.sc_hi;
}

// Q6_K (reference.rs:190-207, :352-386). Lane `sub`: half n = sub/4, positions
// l in [8*lq, 8*lq+8) with lq = sub%4, covering elements 128n + 32k + l (k = 0..3).
struct SbAct6 {
    uint2 a[4];  // 8 codes for each k
    float d;
};
struct SbW6 {
    uint32_t q[4][2];  // unsigned 6-bit codes (0..63), 8 per k
    int sc[4];
    float d;
};
__device__ __forceinline__ void dec_sb_q6k(const uint8_t *base, uint32_t off, int sub, SbW6 &o) {
    const int n = sub >> 2, lq = sub & 3, is = lq >> 1;
    uint32_t A[2], B[2], H[2], S[2], D[1];
    ld_words<2>(base, off + 64 * n + 8 * lq, A);
    ld_words<2>(base, off + 64 * n + 32 + 8 * lq, B);
    ld_words<2>(base, off + 128 + 32 * n + 8 * lq, H);
    ld_words<2>(base, off + 192 + 8 * n, S);
    ld_words<1>(base, off + 208, D);
    o.d = f16_bits_to_f32(D[0]);
#pragma unroll
    for (int k = 0; k < 4; k++) {
#pragma unroll
        for (int w = 0; w < 2; w++) {
            const uint32_t src = (k & 1) ? B[w] : A[w];
            const uint32_t lo4 = (k < 2) ? (src & 0x0F0F0F0Fu) : ((src >> 4) & 0x0F0F0F0Fu);
            o.q[k][w] = lo4 | (((H[w] >> (2 * k)) & 0x03030303u) << 4);
        }
        const int scb = 2 * k + is;  // scale byte index within this half (0..7)
        o.sc[k] = (int)(int8_t)((S[scb >> 2] >> (8 * (scb & 3))) & 0xffu);
    }
}
// Lane share of sumi: sum_k sc_k * (sum q6*a - 32 * sum a), exact.
__device__ __forceinline__ int dot_sb_q6k(const SbW6 &w, const SbAct6 &a) {
    int sumi = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        int acc = dp4a(w.q[k][0], a.a[k].x, 0);
        acc = dp4a(w.q[k][1], a.a[k].y, acc);
        int asum = dp4a(0x01010101u, a.a[k].x, 0);
        asum = dp4a(0x01010101u, a.a[k].y, asum);
        sumi += w.sc[k] * (acc - 32 * asum);
    }
    return sumi;
}

}  // namespace rcu
