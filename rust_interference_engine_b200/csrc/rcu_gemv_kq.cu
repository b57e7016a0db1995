// rcu_gemv_kq.cu -- decode GEMV for ONE activation row over K-quant weights (Q4_K, Q5_K,
// Q6_K x Q8_K activations) with the block dot products on the integer tensor-core path.
// Replaces, for batch 1, the same reference functions as rcu_gemv.cu: matmul_multi /
// compute_rows (kernels/matmul.rs:136-241) driving vec_dot_q4_k / q5_k / q6_k
// (quant/reference.rs:295-386).
//
// Why a second GEMV: the lane-per-block dp4a GEMV issues about 0.2 instructions per weight
// byte (unpacking, scale decoding, activation loads, per-lane combine). At the HBM rate an
// SM receives ~22 bytes per cycle, so that kernel would need close to the SM's 4 issue
// slots per cycle. Here one mma.sync.m16n8k32 (u8 weights x s8 activations) forms the exact
// integer products of 16 rows x 32 weights, and each thread decodes the scales of its own
// sub-blocks only.
//
// Fragment mapping (a warp's thread: g = lane / 4, c = lane % 4):
//   * A holds 16 weight rows (rows g and g + 8 of a 16-row block, as the mma layout puts
//     them in thread (g, c)); A's column chunk c (k = 4c..4c+3 and 16+4c..16+4c+3) carries
//     8 weights of ONE scale group chosen by c: Q4_K / Q5_K sub-block 2c (low nibbles) or
//     2c + 1 (high nibbles); Q6_K the 16-value group (n, m, h) with n = c / 2, h = c % 2;
//   * B is block-diagonal: column j holds the activations of chunk j / 2 and zeros elsewhere
//     (only the threads with c == g / 2 load activations; the others load a zero block), so
//     D[row][2c] = D[row][2c+1] is the exact int32 dot product of chunk c alone.
//     Accumulating D over the steps of a group leaves thread (g, c) with the group's exact
//     sum for rows g and g + 8;
//   * thread c applies the scales / mins of its groups (reference.rs:8-14 unpack, the
//     d * sumi - dmin * summ combine of :295-350, d * sumi of :352-386) in f32; the 4 threads
//     of a row add their partials, then the warps that split the row's superblocks add
//     theirs in a fixed order (deterministic, no atomics on data).
// The per-thread integer pieces add up exactly to the reference's sumi / summ; only the f32
// grouping differs (per thread share instead of per superblock), as in the lane GEMV.
//
// Q4_0 (x Q8_0 activations, vec_dot_q4_0 of quant/reference.rs:221-233) runs on the same tiles:
// eight 18-byte blocks make a 144-byte unit, like a Q4_K superblock. One mma takes one block
// of 16 rows: A's column chunk c carries bytes 4c..4c+3 of the block (weights 4c..4c+3 from
// the low nibbles, 16+4c..16+4c+3 from the high ones), B holds the block's 32 activation codes
// in every column, so every thread ends with the exact int32 sums of its rows g and g + 8.
// Of four consecutive blocks, thread c combines block c: d_w * d_a * (sum - 8 * sum(q_a)),
// the activations' code sum exact (ActsView::sum0).
//
// Shared memory: rows of a stage at a stride = 16 (mod 128), which puts the 16-byte loads of
// a warp's 8 rows in distinct banks. Q6_K superblocks (210 B) are only 2-byte aligned: a
// thread reads its 16 bytes as 4 words in an order rotated by c (word (i + c) % 4 into slot
// i), which spreads those loads over the banks; the activations use the same rotation, so A
// and B agree.
//
// Pipeline: warp 16 is the producer (1-D bulk copies of weight rows into a ring of stages,
// completion on mbarriers, L2 evict-first); warps 0..15 consume. A stage holds 16 * rb rows
// x sl superblocks of one job; the 16 / rb warps of each 16-row block split the slice's
// superblocks (normally one each). A tile is kQG consecutive row groups of one job, so the
// cross-warp reduction runs once per 32 * rb rows: every warp publishes its row partials to
// a shared buffer and the last warp to arrive (shared-memory counter, no barrier) adds them
// in warp order and stores. Activations are read straight from global memory (L1) by the
// threads that use them, before they wait for the stage: no block-wide staging barrier.
// Job descriptors are read into registers once per tile. Every wait is bounded (2 s) and
// reports through the context's error word.
#include <algorithm>
#include <atomic>

#include "rcu_blocks.cuh"
#include "rcu_kernels.h"

namespace rcu {
namespace {

constexpr int kQW = 8;  // consumer warps
constexpr int kQWLog2 = 3;
constexpr int kQThreads = (kQW + 1) * 32;
constexpr int kQG = 2;  // row groups (stages of 16 * rb rows) per tile
constexpr int kQMaxJobs = 96;
constexpr int kQMaxStages = 8;
constexpr int kQRed = 8;  // tile reduction slots; must be >= the number of stages
constexpr uint32_t kQMaxStage = 64 * 1024;
constexpr int kQMaxPeers = 8;

// The zero activation block the threads off B's diagonal read (static device memory is
// zero-initialised).
__device__ __align__(128) uint8_t g_kq_zero[256];

struct KqJob {
    const uint8_t *w;
    float *out;
    const uint32_t *sel;  // indirect (expert) job: weight = w + (*sel) * w_stride
    uint64_t w_stride;
    uint32_t rows, row_bytes, type, tok;
    uint32_t rb_log2;      // 16-row blocks per stage = 1 << rb_log2
    uint32_t sl;           // superblocks per slice (one pipeline stage)
    uint32_t nsl;          // slices per row group
    uint32_t slice_bytes;  // sl * block bytes (a multiple of 16)
    uint32_t pstride;      // shared-memory row stride, = 16 (mod 128)
    uint32_t gpt;          // row groups per tile: kQG, or 1 when half-height tiles balance the CTAs better
    uint32_t tile_begin;
};

// Jobs of one weight type: their tiles [tile0, tile1) go to CTAs [cta0, cta1), so that every
// CTA runs the loop of a single type (one register allocation per type, no spills).
struct KqGroup {
    uint32_t type, job0, job1, tile0, tile1, cta0, cta1;
};
constexpr int kQMaxGroups = 4;

struct KqParams {
    KqJob jobs[kQMaxJobs];
    KqGroup groups[kQMaxGroups];
    int32_t n_jobs, n_groups;
    uint32_t total_tiles, stages, stage_bytes, stage_off;
    uint32_t k, tok0, early_weights;
    ActsView acts;
    uint32_t *err;
    // fused all-reduce push (tensor parallel): outputs also go to ar_dst[q], then each CTA
    // adds its share of kArUnit to every ar_flag[q] (as in rcu_gemv.cu)
    float *ar_dst[kQMaxPeers];
    uint32_t *ar_flag[kQMaxPeers];
    uint32_t ar_ndst, ar_nflag;
    // block-sum capture (the k_gemv_kq<true> instantiation only): every exact per-block
    // integer sum of a row, in the layout of rcu_block_sums, atomically added into
    // dbg[row * dbg_nbs + i]
    int32_t *dbg;
    uint32_t dbg_nbs;
};

struct KqHdr {
    uint64_t full[kQMaxStages];
    uint64_t empty[kQMaxStages];
    int cnt[kQRed];
    float red[kQRed][kQW][kQG][16];  // [tile % kQRed][warp][group][row in the warp's 16-row block]
};
constexpr uint32_t kQHdrBytes = (sizeof(KqHdr) + 127) / 128 * 128;
static_assert(kQRed >= kQMaxStages, "a warp can run up to (stages - 1) tiles ahead");

// The fields of one job the loops use, in registers.
struct JobR {
    const uint8_t *w;
    float *out;
    const uint32_t *sel;
    uint64_t w_stride;
    uint32_t rows, row_bytes, type, tok, rb_log2, sl, nsl, slice_bytes, pstride, gpt, tile_begin;
};
__device__ __forceinline__ void load_job(const KqJob &j, JobR &r) {
    r.w = j.w, r.out = j.out, r.sel = j.sel, r.w_stride = j.w_stride;
    r.rows = j.rows, r.row_bytes = j.row_bytes, r.type = j.type, r.tok = j.tok, r.rb_log2 = j.rb_log2;
    r.sl = j.sl, r.nsl = j.nsl, r.slice_bytes = j.slice_bytes, r.pstride = j.pstride, r.gpt = j.gpt;
    r.tile_begin = j.tile_begin;
}

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ uint4 ldg128(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
__device__ __forceinline__ void words8(const uint4 &x, const uint4 &y, uint32_t (&w)[8]) {
    w[0] = x.x, w[1] = x.y, w[2] = x.z, w[3] = x.w, w[4] = y.x, w[5] = y.y, w[6] = y.z, w[7] = y.w;
}

// One superblock's activations as thread (g, c) feeds them to B, its bsums and scale.
struct ActR {
    uint32_t x[16];  // Q4_K / Q5_K: sub-blocks 2c (x[0..7]) and 2c + 1 (x[8..15]); Q6_K: X[m][i] = x[4m + i]
    uint4 bs;        // Q4_K / Q5_K: pair words 2c, 2c + 1 in .x, .y; Q6_K: pair words 4n .. 4n + 3
    float d;
};

template <int TYPE>
__device__ __forceinline__ void load_act(const int8_t *aq, const float *adk, const uint32_t *abw, uint32_t sb,
                                         uint32_t c, bool bact, ActR &a) {
    if (TYPE == T_Q4_0) {  // unit sb = Q8_0 blocks 8 sb .. 8 sb + 7; adk = d0 row, abw = sum0 row
        const uint8_t *x = reinterpret_cast<const uint8_t *>(aq) + (size_t)sb * QK_K + 4 * c;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            a.x[2 * j] = __ldg(reinterpret_cast<const uint32_t *>(x + 32 * j));
            a.x[2 * j + 1] = __ldg(reinterpret_cast<const uint32_t *>(x + 32 * j + 16));
        }
        a.bs = make_uint4(__float_as_uint(__ldg(adk + 8 * sb + c)), __float_as_uint(__ldg(adk + 8 * sb + 4 + c)),
                          __ldg(abw + 8 * sb + c), __ldg(abw + 8 * sb + 4 + c));
        a.d = 0.0f;
        return;
    }
    a.d = __ldg(adk + sb);
    if (TYPE == T_Q6_K) {
        const uint32_t n = c >> 1, h = c & 1u;
        const uint8_t *xa = bact ? reinterpret_cast<const uint8_t *>(aq) + (size_t)sb * QK_K + 128 * n + 16 * h : g_kq_zero;
#pragma unroll
        for (int m = 0; m < 4; m++)
#pragma unroll
            for (int i = 0; i < 4; i++)
                a.x[4 * m + i] = __ldg(reinterpret_cast<const uint32_t *>(xa + 32 * m + 4u * ((i + c) & 3u)));
        a.bs = ldg128(abw + 8 * sb + 4 * n);
    } else {
        const uint8_t *x = bact ? reinterpret_cast<const uint8_t *>(aq) + (size_t)sb * QK_K + 64 * c : g_kq_zero;
        uint32_t lo[8], hi[8];
        words8(ldg128(x), ldg128(x + 16), lo);
        words8(ldg128(x + 32), ldg128(x + 48), hi);
#pragma unroll
        for (int i = 0; i < 8; i++) a.x[i] = lo[i], a.x[8 + i] = hi[i];
        const uint2 b = __ldg(reinterpret_cast<const uint2 *>(abw + 8 * sb + 2 * c));
        a.bs = make_uint4(b.x, b.y, 0u, 0u);
    }
}

// Q4_K / Q5_K superblock at byte `so` of rows ra (row g) and rb (row g + 8).
template <int TYPE, bool DBG>
__device__ __forceinline__ void kq_q45(const uint8_t *ra, const uint8_t *rb, uint32_t so, const ActR &A, uint32_t c,
                                       float &accA, float &accB, int32_t *dA, int32_t *dB, uint32_t sbg) {
    constexpr uint32_t QO = TYPE == T_Q4_K ? 16 : 48;  // quant bytes (Q5_K: after qh[32])
    const uint8_t *pa = ra + so, *pb = rb + so;
    uint32_t WA[8], WB[8];
    words8(lds128(pa + QO + 32 * c), lds128(pa + QO + 32 * c + 16), WA);
    words8(lds128(pb + QO + 32 * c), lds128(pb + QO + 32 * c + 16), WB);
    uint32_t HA[8], HB[8];
    if (TYPE == T_Q5_K) {
        words8(lds128(pa + 16), lds128(pa + 32), HA);
        words8(lds128(pb + 16), lds128(pb + 32), HB);
    }
    int dl[4] = {0, 0, 0, 0}, dh[4] = {0, 0, 0, 0};
#pragma unroll
    for (int t = 0; t < 4; t++) {
        uint32_t lo[4], hi[4];  // a0 (row g), a1 (row g + 8), a2 (row g), a3 (row g + 8)
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const uint32_t i = 2 * t + (r >> 1);
            const uint32_t w = (r & 1) ? WB[i] : WA[i];
            if (TYPE == T_Q4_K) {
                lo[r] = w & 0x0F0F0F0Fu;
                hi[r] = w & 0xF0F0F0F0u;  // 16 x nibble: the sum is divided by 16 below
            } else {
                const uint32_t hb = (r & 1) ? HB[i] : HA[i];
                lo[r] = (w & 0x0F0F0F0Fu) | (((hb >> (2 * c)) & 0x01010101u) << 4);
                hi[r] = ((w >> 4) & 0x0F0F0F0Fu) | (((hb >> (2 * c + 1)) & 0x01010101u) << 4);
            }
        }
        mma_u8s8(dl, lo[0], lo[1], lo[2], lo[3], A.x[2 * t], A.x[2 * t + 1]);
        mma_u8s8(dh, hi[0], hi[1], hi[2], hi[3], A.x[8 + 2 * t], A.x[8 + 2 * t + 1]);
    }
    // scales of sub-blocks 2c, 2c + 1 and their mins (get_scale_min_k4, reference.rs:8-14)
    const uint32_t sh = 16u * (c & 1u);
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const uint4 hd = lds128(r ? pb : pa);
        const uint32_t a = hd.y >> sh, b = hd.w >> sh, cc = hd.z >> sh;
        const uint32_t scp = c < 2 ? a : ((b & 0x0F0Fu) | ((a >> 2) & 0x3030u));
        const uint32_t mnp = c < 2 ? cc : (((b >> 4) & 0x0F0Fu) | ((cc >> 2) & 0x3030u));
        const int s_lo = dl[2 * r], s_hi = TYPE == T_Q4_K ? (dh[2 * r] >> 4) : dh[2 * r];
        const int I = (int)(scp & 63u) * s_lo + (int)((scp >> 8) & 63u) * s_hi;
        const int M = dp2a_lo(A.bs.x, (mnp & 63u) * 0x0101u, dp2a_lo(A.bs.y, ((mnp >> 8) & 63u) * 0x0101u, 0));
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hd.x));
        float &acc = r ? accB : accA;
        acc = fmaf(A.d, fmaf(-f.y, (float)M, f.x * (float)I), acc);
        if constexpr (DBG) {
            if (int32_t *d = r ? dB : dA) {
                atomicAdd(d + 2 * sbg, I);
                atomicAdd(d + 2 * sbg + 1, M);
            }
        }
    }
}

// Q6_K value of group m (0..3) for 4 weights: low nibble from ql word l0 (m = 0, 2) or l1
// (m = 1, 3), high 2 bits from qh word hh (reference.rs:190-207).
template <int M>
__device__ __forceinline__ uint32_t q6v(uint32_t l0, uint32_t l1, uint32_t hh) {
    if (M == 0) return (l0 & 0x0F0F0F0Fu) | ((hh << 4) & 0x30303030u);
    if (M == 1) return (l1 & 0x0F0F0F0Fu) | ((hh << 2) & 0x30303030u);
    if (M == 2) return ((l0 >> 4) & 0x0F0F0F0Fu) | (hh & 0x30303030u);
    return ((l1 >> 4) & 0x0F0F0F0Fu) | ((hh >> 2) & 0x30303030u);
}

// 16 bytes at byte offset `off` of a row (row start 16-aligned, off even) as 4 words, slot
// i <- word (i + c) % 4. A4: off is a multiple of 4.
template <bool A4>
__device__ __forceinline__ void ld4_rot(const uint8_t *row, uint32_t off, uint32_t c, uint32_t (&o)[4]) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t wo = off + 4u * ((i + c) & 3u);
        o[i] = A4 ? *reinterpret_cast<const uint32_t *>(row + wo) : lds_u32_at(row, wo);
    }
}

// Q6_K superblock at byte `so` of rows ra / rb (A4: so is a multiple of 4, i.e. an even
// superblock index within the slice).
template <bool A4, bool DBG>
__device__ __forceinline__ void kq_q6(const uint8_t *ra, const uint8_t *rb, uint32_t so, const ActR &A, uint32_t c,
                                      float &accA, float &accB, int32_t *dA, int32_t *dB, uint32_t sbg) {
    const uint32_t n = c >> 1, h = c & 1u;
    uint32_t LA0[4], LA1[4], HA[4], LB0[4], LB1[4], HB[4];
    ld4_rot<A4>(ra, so + 64 * n + 16 * h, c, LA0);
    ld4_rot<A4>(ra, so + 64 * n + 32 + 16 * h, c, LA1);
    ld4_rot<A4>(ra, so + 128 + 32 * n + 16 * h, c, HA);
    ld4_rot<A4>(rb, so + 64 * n + 16 * h, c, LB0);
    ld4_rot<A4>(rb, so + 64 * n + 32 + 16 * h, c, LB1);
    ld4_rot<A4>(rb, so + 128 + 32 * n + 16 * h, c, HB);
    int D[4][4];
#pragma unroll
    for (int m = 0; m < 4; m++) D[m][0] = D[m][1] = D[m][2] = D[m][3] = 0;
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const int i0 = 2 * u, i1 = 2 * u + 1;
        mma_u8s8(D[0], q6v<0>(LA0[i0], LA1[i0], HA[i0]), q6v<0>(LB0[i0], LB1[i0], HB[i0]),
                 q6v<0>(LA0[i1], LA1[i1], HA[i1]), q6v<0>(LB0[i1], LB1[i1], HB[i1]), A.x[i0], A.x[i1]);
        mma_u8s8(D[1], q6v<1>(LA0[i0], LA1[i0], HA[i0]), q6v<1>(LB0[i0], LB1[i0], HB[i0]),
                 q6v<1>(LA0[i1], LA1[i1], HA[i1]), q6v<1>(LB0[i1], LB1[i1], HB[i1]), A.x[4 + i0], A.x[4 + i1]);
        mma_u8s8(D[2], q6v<2>(LA0[i0], LA1[i0], HA[i0]), q6v<2>(LB0[i0], LB1[i0], HB[i0]),
                 q6v<2>(LA0[i1], LA1[i1], HA[i1]), q6v<2>(LB0[i1], LB1[i1], HB[i1]), A.x[8 + i0], A.x[8 + i1]);
        mma_u8s8(D[3], q6v<3>(LA0[i0], LA1[i0], HA[i0]), q6v<3>(LB0[i0], LB1[i0], HB[i0]),
                 q6v<3>(LA0[i1], LA1[i1], HA[i1]), q6v<3>(LB0[i1], LB1[i1], HB[i1]), A.x[12 + i0], A.x[12 + i1]);
    }
    // q6 - 32: subtract 32 x the group's activation sum (Q8_K bsums are per 16 values, one
    // per Q6_K scale group); groups 8n + 2m + h are the halves h of pair words 4n + m
    const uint32_t bw[4] = {A.bs.x, A.bs.y, A.bs.z, A.bs.w};
    int bs[4];
#pragma unroll
    for (int m = 0; m < 4; m++) bs[m] = h ? ((int)bw[m] >> 16) : (int)(int16_t)(bw[m] & 0xffffu);
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const uint8_t *row = r ? rb : ra;
        uint32_t S0, S1;  // scales[8n .. 8n + 7]; group m's scale is byte h + 2m
        if (A4) {
            S0 = *reinterpret_cast<const uint32_t *>(row + so + 192 + 8 * n);
            S1 = *reinterpret_cast<const uint32_t *>(row + so + 196 + 8 * n);
        } else {
            S0 = lds_u32_at(row, so + 192 + 8 * n);
            S1 = lds_u32_at(row, so + 196 + 8 * n);
        }
        int I = 0;
#pragma unroll
        for (int m = 0; m < 4; m++) {
            const int sc = sbyte((m & 2) ? S1 : S0, h + 2 * (m & 1));
            I += sc * (D[m][2 * r] - 32 * bs[m]);
        }
        const uint32_t db = *reinterpret_cast<const uint16_t *>(row + so + 208);
        float &acc = r ? accB : accA;
        acc = fmaf(f16_bits_to_f32(db) * A.d, (float)I, acc);
        if constexpr (DBG) {
            if (int32_t *d = r ? dB : dA) atomicAdd(d + sbg, I);
        }
    }
}

// Q4_0 unit (8 blocks) at byte `so` of rows ra / rb.
template <bool DBG>
__device__ __forceinline__ void kq_q40(const uint8_t *ra, const uint8_t *rb, uint32_t so, const ActR &A, uint32_t c,
                                       float &accA, float &accB, int32_t *dA, int32_t *dB, uint32_t sbg) {
#pragma unroll
    for (int s4 = 0; s4 < 2; s4++) {
        int D[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t b = 4 * s4 + j, off = so + 18 * b + 2 + 4 * c;  // 4-aligned for odd blocks
            const uint32_t wa = (b & 1) ? *reinterpret_cast<const uint32_t *>(ra + off) : lds_u32_at(ra, off);
            const uint32_t wb = (b & 1) ? *reinterpret_cast<const uint32_t *>(rb + off) : lds_u32_at(rb, off);
            D[j][0] = D[j][1] = D[j][2] = D[j][3] = 0;
            mma_u8s8(D[j], wa & 0x0F0F0F0Fu, wb & 0x0F0F0F0Fu, (wa >> 4) & 0x0F0F0F0Fu, (wb >> 4) & 0x0F0F0F0Fu,
                     A.x[2 * b], A.x[2 * b + 1]);
        }
        // this thread's block of the four: 4 s4 + c
        const int sg = c == 0 ? D[0][0] : c == 1 ? D[1][0] : c == 2 ? D[2][0] : D[3][0];
        const int sh = c == 0 ? D[0][2] : c == 1 ? D[1][2] : c == 2 ? D[2][2] : D[3][2];
        const uint32_t bo = so + 18 * (4 * s4 + c);
        const float da = __uint_as_float(s4 ? A.bs.y : A.bs.x);
        const int sa8 = 8 * (int)(s4 ? A.bs.w : A.bs.z);
        const float dwa = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(ra + bo));
        const float dwb = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(rb + bo));
        accA = fmaf(dwa * da, (float)(sg - sa8), accA);
        accB = fmaf(dwb * da, (float)(sh - sa8), accB);
        if constexpr (DBG) {  // Q8_0 block 8 unit + 4 s4 + c
            if (dA) atomicAdd(dA + 8 * sbg + 4 * s4 + c, sg - sa8);
            if (dB) atomicAdd(dB + 8 * sbg + 4 * s4 + c, sh - sa8);
        }
    }
}

// Unit sbl of the stage's slice (sbg: the unit's index in the row, for the block-sum capture).
template <int TYPE, bool DBG>
__device__ __forceinline__ void kq_block(const uint8_t *ra, const uint8_t *rb, uint32_t sbl, const ActR &A, uint32_t c,
                                         float &accA, float &accB, int32_t *dA, int32_t *dB, uint32_t sbg) {
    constexpr uint32_t BB = TYPE == T_Q4_K || TYPE == T_Q4_0 ? 144 : TYPE == T_Q5_K ? 176 : 210;
    if (TYPE == T_Q4_0) {
        kq_q40<DBG>(ra, rb, sbl * BB, A, c, accA, accB, dA, dB, sbg);
    } else if (TYPE == T_Q6_K) {
        if (sbl & 1u)
            kq_q6<false, DBG>(ra, rb, sbl * BB, A, c, accA, accB, dA, dB, sbg);
        else
            kq_q6<true, DBG>(ra, rb, sbl * BB, A, c, accA, accB, dA, dB, sbg);
    } else {
        kq_q45<TYPE, DBG>(ra, rb, sbl * BB, A, c, accA, accB, dA, dB, sbg);
    }
}

struct Ring {  // consumer-side stage ring position
    uint32_t s, ph;
};

// The stages of one tile for one consumer warp: kQG row groups x nsl slices; this warp's
// superblocks of each slice are part, part + wpb, ... (< sl), taken two at a time with
// independent accumulators (two mma chains in flight) and their activations loaded before
// the stage wait. Row partials of group gi end in accA[gi] (row g of the warp's 16-row
// block) / accB[gi] (row g + 8).
template <int TYPE, bool DBG>
__device__ __forceinline__ bool kq_tile(const KqParams &p, KqHdr *h, uint8_t *stages, const JobR &J, uint32_t ngrp,
                                        bool skip, const int8_t *aq, const float *adk, const uint32_t *abw,
                                        uint32_t rbk, uint32_t part, uint32_t wpb, uint32_t g, uint32_t c, bool bact,
                                        uint32_t lane, Ring &R, float (&accA)[kQG], float (&accB)[kQG], uint32_t r0) {
    const uint32_t S = p.stages;
    const uint32_t rofs = (rbk * 16u + g) * J.pstride;
#pragma unroll
    for (int gi = 0; gi < kQG; gi++) {
        if ((uint32_t)gi >= ngrp) break;
        float a1 = 0.0f, b1 = 0.0f;  // second chain
        int32_t *dA = nullptr, *dB = nullptr;  // block-sum capture rows (rows of the tile only)
        if constexpr (DBG) {
            const uint32_t row = r0 + gi * (16u << J.rb_log2) + rbk * 16u + g;
            if (row < J.rows) dA = p.dbg + (uint64_t)row * p.dbg_nbs;
            if (row + 8 < J.rows) dB = p.dbg + (uint64_t)(row + 8) * p.dbg_nbs;
        }
        for (uint32_t sli = 0; sli < J.nsl; sli++) {
            const uint32_t sb0 = sli * J.sl;
            uint32_t sbl = part;
            ActR A0, A1;
            const bool two = sbl + wpb < J.sl;
            if (!skip) {
                load_act<TYPE>(aq, adk, abw, sb0 + sbl, c, bact, A0);
                if (two) load_act<TYPE>(aq, adk, abw, sb0 + sbl + wpb, c, bact, A1);
            }
            if (!mbar_wait_bounded(&h->full[R.s], R.ph, p.err, ERR_TIMEOUT_FULL)) return false;
            if (!skip) {
                const uint8_t *ra = stages + R.s * p.stage_bytes + rofs;
                const uint8_t *rb = ra + 8u * J.pstride;
                if (two) {
                    kq_block<TYPE, DBG>(ra, rb, sbl, A0, c, accA[gi], accB[gi], dA, dB, sb0 + sbl);
                    kq_block<TYPE, DBG>(ra, rb, sbl + wpb, A1, c, a1, b1, dA, dB, sb0 + sbl + wpb);
                    sbl += 2 * wpb;
                } else {
                    kq_block<TYPE, DBG>(ra, rb, sbl, A0, c, accA[gi], accB[gi], dA, dB, sb0 + sbl);
                    sbl += wpb;
                }
                for (; sbl < J.sl; sbl += wpb) {  // slices wider than two superblocks per warp
                    load_act<TYPE>(aq, adk, abw, sb0 + sbl, c, bact, A0);
                    kq_block<TYPE, DBG>(ra, rb, sbl, A0, c, a1, b1, dA, dB, sb0 + sbl);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&h->empty[R.s]);
            if (++R.s == S) {
                R.s = 0;
                R.ph ^= 1u;
            }
        }
        accA[gi] += a1;
        accB[gi] += b1;
    }
    return true;
}

__device__ __forceinline__ void kq_store(const KqParams &p, float *out, uint32_t row, float v) {
    out[row] = v;
    for (uint32_t q = 0; q < p.ar_ndst; q++) p.ar_dst[q][row] = v;
}

// Consumer warps of a CTA whose tiles all hold weights of type TYPE.
template <int TYPE, bool DBG>
__device__ __forceinline__ void kq_consume(const KqParams &p, KqHdr *h, uint8_t *stages, const KqGroup &G, int warp,
                                           int lane) {
    const uint32_t g = lane >> 2, c = lane & 3;
    const bool bact = c == (g >> 1);
    const ActsView &AV = p.acts;
    const uint32_t k = p.k, nsb = k / QK_K;
    Ring R{0, 0};
    uint32_t tloc = 0;
    int ji = (int)G.job0 - 1;
    JobR J{};
    uint32_t next_begin = 0;
    const uint32_t step = G.cta1 - G.cta0;
    for (uint32_t tile = G.tile0 + (blockIdx.x - G.cta0); tile < G.tile1; tile += step, tloc++) {
        while (ji + 1 < (int)G.job1 && next_begin <= tile) {
            load_job(p.jobs[++ji], J);
            next_begin = ji + 1 < (int)G.job1 ? p.jobs[ji + 1].tile_begin : 0xffffffffu;
        }
        const uint32_t wpb = kQW >> J.rb_log2, rbk = warp >> (kQWLog2 - J.rb_log2), part = warp & (wpb - 1);
        const uint32_t grows = 16u << J.rb_log2, r0 = (tile - J.tile_begin) * (J.gpt * grows);
        const uint32_t ngrp = min(J.gpt, (J.rows - r0 + grows - 1) / grows);
        const uint32_t ex = J.sel ? *(volatile const uint32_t *)J.sel : 0u;
        const bool skip = ex == kNoExpert;
        const uint64_t trow = (uint64_t)p.tok0 + J.tok;
        // Q8_K rows (codes, superblock scales, bsum pairs) or, for Q4_0, Q8_0 rows (codes, block
        // scales, exact code sums)
        const int8_t *aq = TYPE == T_Q4_0 ? AV.q0 + trow * k : AV.qk + trow * k;
        const float *adk = TYPE == T_Q4_0 ? AV.d0 + trow * (k / QK) : AV.dk + trow * nsb;
        const uint32_t *abw = TYPE == T_Q4_0 ? reinterpret_cast<const uint32_t *>(AV.sum0 + trow * (k / QK))
                                             : reinterpret_cast<const uint32_t *>(AV.bsk + trow * (k / 16));
        float accA[kQG], accB[kQG];
#pragma unroll
        for (int gi = 0; gi < kQG; gi++) accA[gi] = accB[gi] = 0.0f;
        if (!kq_tile<TYPE, DBG>(p, h, stages, J, ngrp, skip, aq, adk, abw, rbk, part, wpb, g, c, bact, lane, R, accA,
                                accB, r0))
            return;
        // tile done: the 4 threads of each row add their shares, every warp publishes its rows'
        // partials; the last warp to arrive adds the parts in warp order and stores
        const uint32_t ri = tloc % kQRed;
#pragma unroll
        for (int gi = 0; gi < kQG; gi++) {
            float a = accA[gi], b = accB[gi];
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            a += __shfl_xor_sync(0xffffffffu, a, 2);
            b += __shfl_xor_sync(0xffffffffu, b, 1);
            b += __shfl_xor_sync(0xffffffffu, b, 2);
            if (c == 0) {
                h->red[ri][warp][gi][g] = a;
                h->red[ri][warp][gi][g + 8] = b;
            }
        }
        __syncwarp();
        __threadfence_block();
        int old = 0;
        if (lane == 0) old = atomicAdd(&h->cnt[ri], 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == kQW - 1) {
            __threadfence_block();
            if (!skip) {
                const uint32_t nrows = min(ngrp * grows, J.rows - r0);
                for (uint32_t i = lane; i < nrows; i += 32) {
                    const uint32_t gi = i >> (4 + J.rb_log2), ii = i & (grows - 1), bk = ii >> 4, rr = ii & 15u;
                    float v = 0.0f;
                    for (uint32_t q = 0; q < wpb; q++) v += *((volatile float *)&h->red[ri][bk * wpb + q][gi][rr]);
                    kq_store(p, J.out, r0 + i, v);
                }
            }
            __syncwarp();
            if (lane == 0) atomicExch(&h->cnt[ri], 0);
        }
        __syncwarp();
    }
}

template <bool DBG>
__global__ void __launch_bounds__(kQThreads, 1) k_gemv_kq(const __grid_constant__ KqParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    KqHdr *h = reinterpret_cast<KqHdr *>(smem);
    uint8_t *stages = smem + p.stage_off;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t S = p.stages;
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; s++) {
            mbar_init(&h->full[s], 1);
            mbar_init(&h->empty[s], kQW);
        }
        fence_mbar_init();
    }
    if (threadIdx.x < kQRed) h->cnt[threadIdx.x] = 0;
    __syncthreads();
    int gq = 0;
    while (gq + 1 < p.n_groups && blockIdx.x >= p.groups[gq].cta1) gq++;
    const KqGroup &G = p.groups[gq];

    if (warp == kQW) {  // ---- producer: one bulk copy per weight row and slice ----
        if (!p.early_weights) pdl_wait();
        const uint64_t pol = policy_evict_first();
        uint32_t li = 0, s = 0, ph = 0;  // stages issued, ring slot, pass parity
        int ji = (int)G.job0 - 1;
        JobR J{};
        uint32_t next_begin = 0;
        bool ok = true;
        const uint32_t step = G.cta1 - G.cta0;
        for (uint32_t tile = G.tile0 + (blockIdx.x - G.cta0); ok && tile < G.tile1; tile += step) {
            while (ji + 1 < (int)G.job1 && next_begin <= tile) {
                load_job(p.jobs[++ji], J);
                next_begin = ji + 1 < (int)G.job1 ? p.jobs[ji + 1].tile_begin : 0xffffffffu;
            }
            const uint32_t grows = 16u << J.rb_log2, r0 = (tile - J.tile_begin) * (J.gpt * grows);
            const uint32_t ex = J.sel ? *(volatile const uint32_t *)J.sel : 0u;
            for (uint32_t gi = 0; ok && gi < J.gpt && r0 + gi * grows < J.rows; gi++) {
                const uint32_t g0 = r0 + gi * grows, nrows = min(grows, J.rows - g0);
                for (uint32_t sl = 0; sl < J.nsl; sl++) {
                    if (li >= S) {
                        int w_ok = 1;
                        if (lane == 0) w_ok = mbar_wait_bounded(&h->empty[s], ph ^ 1u, p.err, ERR_TIMEOUT_EMPTY);
                        if (!__shfl_sync(0xffffffffu, w_ok, 0)) {
                            ok = false;
                            break;
                        }
                    }
                    if (ex == kNoExpert) {  // routed to another rank's expert: nothing to load
                        if (lane == 0) mbar_arrive(&h->full[s]);
                    } else {
                        const uint8_t *src = J.w + (uint64_t)ex * J.w_stride + (uint64_t)g0 * J.row_bytes +
                                             (uint64_t)sl * J.slice_bytes;
                        uint8_t *dst = stages + s * p.stage_bytes;
                        if (lane == 0) mbar_arrive_expect_tx(&h->full[s], nrows * J.slice_bytes);
                        __syncwarp();
                        for (uint32_t r = lane; r < nrows; r += 32)
                            bulk_g2s(dst + r * J.pstride, src + (uint64_t)r * J.row_bytes, J.slice_bytes, &h->full[s],
                                     pol);
                    }
                    li++;
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
        }
        // never leave the CTA with copies in flight: wait for the last phase of each stage
        if (lane == 0) {
            for (uint32_t st = 0; st < S && st < li; st++) {
                const uint32_t last = ((li - 1 - st) / S) * S + st;
                mbar_wait_bounded(&h->full[st], (last / S) & 1u, p.err, ERR_TIMEOUT_DRAIN);
            }
        }
        return;
    }

    // ---- consumers ----
    pdl_wait();  // the activations come from the kernel before this one
    switch (G.type) {
        case T_Q4_K: kq_consume<T_Q4_K, DBG>(p, h, stages, G, warp, lane); break;
        case T_Q5_K: kq_consume<T_Q5_K, DBG>(p, h, stages, G, warp, lane); break;
        case T_Q4_0: kq_consume<T_Q4_0, DBG>(p, h, stages, G, warp, lane); break;
        default: kq_consume<T_Q6_K, DBG>(p, h, stages, G, warp, lane); break;
    }
    if (p.ar_nflag) {  // this CTA's rows are in every receive buffer: count it in
        __threadfence_system();
        named_bar_sync(1, kQW * 32);
        const uint32_t add = blockIdx.x == 0 ? kArUnit - (gridDim.x - 1) : 1u;
        if (threadIdx.x == 0)
            for (uint32_t q = 0; q < p.ar_nflag; q++) atomicAdd_system(p.ar_flag[q], add);
    }
}

uint32_t round_up_u(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

// Tiling of one job: slice length sl (a divisor of the superblock count; Q6_K slices a
// multiple of 8 superblocks so that 210-byte rows stay 16-byte multiples), 16-row blocks per
// stage rb (so that the kQW / rb warps of a block have a superblock each), stage bytes
// <= 64 KB. Prefers slices the block's warps split evenly, then slices of two superblocks
// per warp (two independent chains), then longer slices.
bool kq_plan(const rcu_weight *w, uint32_t k, KqJob &jd) {
    const int t = w->type;
    if (t != T_Q4_K && t != T_Q5_K && t != T_Q6_K && t != T_Q4_0) return false;
    if (w->cols != k || k % QK_K != 0 || w->row_bytes % 16 != 0 || ((uintptr_t)w->data & 15u)) return false;
    // units of 256 values: a K-quant superblock, or eight Q4_0 blocks (144 bytes)
    const uint32_t bb = t == T_Q4_0 ? 8u * 18u : (uint32_t)block_bytes(t), nsb = k / QK_K;
    double best = -1.0;
    for (uint32_t sl = nsb; sl >= 1; sl--) {
        if (nsb % sl || (sl * bb) % 16) continue;
        uint32_t ps = sl * bb;
        ps += (16u + 128u - ps % 128u) % 128u;
        uint32_t rbl0 = 0;
        while ((uint32_t)(kQW >> rbl0) > sl && rbl0 < (uint32_t)kQWLog2) rbl0++;
        // taller stages (more 16-row blocks, fewer warps per block) give each warp two units
        for (uint32_t rbl = rbl0; rbl <= (uint32_t)kQWLog2; rbl++) {
            if ((16u << rbl) * ps > kQMaxStage) break;
            const uint32_t wpb = kQW >> rbl, per = (sl + wpb - 1) / wpb;
            const double bal = (double)sl / (double)(wpb * per);
            const double score = bal * 8.0 + (per == 2 ? 2.0 : 0.0) + (double)sl / nsb - 0.01 * rbl;
            if (score > best) {
                best = score;
                jd.sl = sl;
                jd.rb_log2 = rbl;
                jd.pstride = ps;
            }
        }
    }
    if (best < 0.0) return false;
    jd.nsl = nsb / jd.sl;
    jd.slice_bytes = jd.sl * bb;
    jd.type = (uint32_t)t;
    jd.row_bytes = (uint32_t)w->row_bytes;
    return true;
}

uint32_t kq_stage_bytes(const KqJob &jd) { return round_up_u((16u << jd.rb_log2) * jd.pstride, 128); }

// Shared-memory layout: header, then the weight stages. False when two stages do not fit.
bool kq_smem_layout(const rcu_ctx *ctx, uint32_t stage_bytes, KqParams &p) {
    p.stage_off = kQHdrBytes;
    const uint32_t budget = (uint32_t)ctx->max_smem_optin;
    if (p.stage_off + 2 * stage_bytes > budget) return false;
    p.stages = std::min<uint32_t>(kQMaxStages, (budget - p.stage_off) / stage_bytes);
    return true;
}

}  // namespace

static bool kq_ok(const rcu_ctx *ctx, uint32_t k, uint32_t have, const HostJob *jobs, int n_jobs);

bool gemv_kq_ok(const rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs) {
    return kq_ok(ctx, a.k, a.have, jobs, n_jobs);
}

static bool kq_ok(const rcu_ctx *ctx, uint32_t k, uint32_t have, const HostJob *jobs, int n_jobs) {
    if (!ctx->gemv_kq || n_jobs < 1 || n_jobs > kQMaxJobs) return false;
    for (int i = 0; i < n_jobs; i++)
        if (!(have & act_format(jobs[i].w->type))) return false;
    // Q4_0 rows shorter than 4096 values stay on the lane GEMV, which measured faster there
    // (config 1, 6144 x 2048: 3.5 vs 2.8 TB/s; 2 x 28672 x 8192: 2.7 vs 3.8 TB/s here)
    for (int i = 0; i < n_jobs; i++)
        if (jobs[i].w->type == T_Q4_0 && k < ctx->gemv_kq_q4_0_min_k) return false;
    uint64_t bytes = 0;
    uint32_t stage_bytes = 0;
    for (int i = 0; i < n_jobs; i++) {
        KqJob jd{};
        if (!kq_plan(jobs[i].w, k, jd)) return false;
        if (jobs[i].sel && jobs[i].w_stride % 16 != 0) return false;
        bytes += (uint64_t)(jobs[i].rows ? jobs[i].rows : jobs[i].w->rows) * jobs[i].w->row_bytes;
        stage_bytes = std::max(stage_bytes, kq_stage_bytes(jd));
    }
    KqParams lay;
    if (!kq_smem_layout(ctx, stage_bytes, lay)) return false;
    // Small launches take the lane GEMV: with 1-2 tiles per CTA this kernel's start-up is not
    // hidden; K = 768 expert rows also give it few tiles.
    return bytes >= ctx->gemv_kq_min_bytes;
}

int launch_gemv_kq(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs, uint32_t tok0,
                   const ArPush *push) {
    KqParams p{};
    p.n_jobs = n_jobs;
    p.k = a.k;
    p.tok0 = tok0;
    p.acts = a;
    p.err = ctx->dev_err;
    p.early_weights = ctx->early_weights ? 1u : 0u;
    if (push) {
        if (n_jobs != 1 || tok0 != 0 || push->n_dst > kQMaxPeers || push->n_flag > kQMaxPeers)
            return set_err(ctx, RCU_ERR_INVALID, "gemv: all-reduce push needs one job, one launch, <= 8 ranks");
        p.ar_ndst = push->n_dst;
        p.ar_nflag = push->n_flag;
        for (uint32_t q = 0; q < push->n_dst; q++) p.ar_dst[q] = push->dst[q];
        for (uint32_t q = 0; q < push->n_flag; q++) p.ar_flag[q] = push->flag[q];
    }
    // jobs grouped by weight type (each group's tiles run on CTAs of their own)
    uint32_t tiles = 0, stage_bytes = 0;
    uint64_t gbytes[kQMaxGroups] = {};
    int nj = 0;
    for (const int ty : {T_Q4_K, T_Q5_K, T_Q6_K, T_Q4_0}) {
        KqGroup &G = p.groups[p.n_groups];
        G.type = (uint32_t)ty;
        G.job0 = (uint32_t)nj;
        G.tile0 = tiles;
        for (int i = 0; i < n_jobs; i++) {
            if (jobs[i].w->type != ty) continue;
            KqJob &jd = p.jobs[nj++];
            if (!kq_plan(jobs[i].w, a.k, jd))
                return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemv: weight not K-quant tileable");
            jd.w = jobs[i].w->data;
            jd.out = jobs[i].out + (jobs[i].sel ? 0 : (uint64_t)tok0 * jobs[i].ld);  // indirect jobs: own rows
            jd.sel = jobs[i].sel;
            jd.w_stride = jobs[i].w_stride;
            jd.tok = jobs[i].tok;
            jd.rows = jobs[i].rows ? jobs[i].rows : (uint32_t)jobs[i].w->rows;
            if (jd.sel) p.early_weights = 0;  // the producer reads the router's choice: wait first
            jd.gpt = kQG;
            jd.tile_begin = tiles;
            const uint32_t trows = kQG * (16u << jd.rb_log2);
            tiles += (jd.rows + trows - 1) / trows;
            stage_bytes = std::max(stage_bytes, kq_stage_bytes(jd));
            gbytes[p.n_groups] += (uint64_t)jd.rows * jd.row_bytes;
        }
        G.job1 = (uint32_t)nj;
        G.tile1 = tiles;
        if (G.job1 > G.job0) p.n_groups++;
    }
    if (nj != n_jobs) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemv: weight not K-quant tileable");
    // CTAs per group in proportion to its bytes (at least one, at most one per tile)
    uint64_t total_bytes = 0;
    for (int q = 0; q < p.n_groups; q++) total_bytes += gbytes[q];
    const uint32_t sms = std::max<uint32_t>((uint32_t)ctx->num_sms, (uint32_t)p.n_groups);
    uint32_t cta = 0;
    for (int q = 0; q < p.n_groups; q++) {
        KqGroup &G = p.groups[q];
        const uint32_t gt = G.tile1 - G.tile0;
        uint32_t n = q + 1 == p.n_groups ? sms - cta
                                         : (uint32_t)((double)sms * (double)gbytes[q] / (double)std::max<uint64_t>(total_bytes, 1) + 0.5);
        n = std::max<uint32_t>(1u, std::min<uint32_t>(n, gt));
        n = std::min<uint32_t>(n, sms - cta - (uint32_t)(p.n_groups - 1 - q));  // leave one for each group after
        G.cta0 = cta;
        G.cta1 = cta + n;
        cta += n;
    }
    // A group whose CTAs get one or two tiles balances better with half-height tiles when that
    // shortens the longest CTA's share (e.g. 160 tiles on 115 CTAs: 2 tiles; 320 half tiles: 3
    // halves); tile numbers are then assigned again. (With more tiles per CTA the extra
    // per-tile reductions cost more than the balance gains: measured on the gate+up launch.)
    tiles = 0;
    for (int q = 0; q < p.n_groups; q++) {
        KqGroup &G = p.groups[q];
        const uint32_t n = G.cta1 - G.cta0;
        uint32_t t2 = 0, t1 = 0;
        for (uint32_t j = G.job0; j < G.job1; j++) {
            const uint32_t grows = 16u << p.jobs[j].rb_log2;
            t2 += (p.jobs[j].rows + kQG * grows - 1) / (kQG * grows);
            t1 += (p.jobs[j].rows + grows - 1) / grows;
        }
        const uint32_t full = (t2 + n - 1) / n;  // the longest CTA's share in full tiles
        const uint32_t gpt = full <= 2 && (t1 + n - 1) / n < kQG * full ? 1u : (uint32_t)kQG;
        G.tile0 = tiles;
        for (uint32_t j = G.job0; j < G.job1; j++) {
            KqJob &jd = p.jobs[j];
            jd.gpt = gpt;
            jd.tile_begin = tiles;
            const uint32_t trows = gpt * (16u << jd.rb_log2);
            tiles += (jd.rows + trows - 1) / trows;
        }
        G.tile1 = tiles;
    }
    p.total_tiles = tiles;
    p.stage_bytes = stage_bytes;
    if (!kq_smem_layout(ctx, stage_bytes, p))
        return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemv: two weight stages exceed shared memory");
    const uint32_t smem_bytes = p.stage_off + p.stages * stage_bytes;
    const uint32_t grid = cta;
    if (push && grid > kArUnit) return set_err(ctx, RCU_ERR_INVALID, "gemv: grid above the all-reduce counter unit");
    const bool dbg = ctx->dbg_sums != nullptr;
    if (dbg) {
        if (n_jobs != 1 || push) return set_err(ctx, RCU_ERR_INVALID, "block-sum capture: one job, no push");
        p.dbg = ctx->dbg_sums;
        p.dbg_nbs = ctx->dbg_nbs;
    }
    auto kern = dbg ? k_gemv_kq<true> : k_gemv_kq<false>;
    static std::atomic<bool> attr_set[2][64] = {};  // per instantiation and device; contexts may live on several threads
    std::atomic<bool> &set = attr_set[dbg ? 1 : 0][ctx->device & 63];
    if (!set.load(std::memory_order_acquire)) {
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)ctx->max_smem_optin));
        set.store(true, std::memory_order_release);
    }
    RCU_CUDA_TRY(ctx, launch_k(ctx, kern, dim3(grid), dim3(kQThreads), smem_bytes, p));
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

}  // namespace rcu
