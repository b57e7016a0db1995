// rcu_gemv_kq.cu -- decode GEMV for ONE activation row over K-quant weights (Q4_K, Q5_K,
// Q6_K x Q8_K activations) with the block dot products on the integer tensor-core path.
// Replaces, for batch 1, the same reference functions as rcu_gemv.cu: matmul_multi /
// compute_rows (kernels/matmul.rs:136-241) driving vec_dot_q4_k / q5_k / q6_k
// (quant/reference.rs:295-386).
//
// Why a second GEMV: the lane-per-block dp4a GEMV issues about 0.2 instructions per weight
// byte (unpacking, scale decoding, activation loads, per-lane combine). At the HBM rate an
// SM receives ~24 bytes per cycle, so that kernel would need more than the SM's 4 issue
// slots per cycle. Here one mma.sync.m16n8k32 (u8 weights x s8 activations) forms the exact
// integer products of 16 rows x 32 weights, and each thread decodes the scales of its own
// sub-blocks only: about 0.05 (Q4_K) / 0.07 (Q6_K) instructions per byte.
//
// Fragment mapping (a warp's thread: g = lane / 4, c = lane % 4):
//   * A holds 16 weight rows (rows g and g + 8 of a 16-row block, as the mma layout puts
//     them in thread (g, c)); A's column chunk c (k = 4c..4c+3 and 16+4c..16+4c+3) carries
//     8 weights of ONE scale group chosen by c: Q4_K / Q5_K sub-block 2c (low nibbles) or
//     2c + 1 (high nibbles); Q6_K the 16-value group (n, m, h) with n = c / 2, h = c % 2;
//   * B is block-diagonal: column j holds the activations of chunk j / 2 and zeros elsewhere
//     (only the threads with c == g / 2 load activations), so D[row][2c] = D[row][2c+1] is
//     the exact int32 dot product of chunk c alone. Accumulating D over the steps of a group
//     leaves thread (g, c) with the group's exact sum for rows g and g + 8;
//   * thread c applies the scales / mins of its groups (reference.rs:8-14 unpack, the
//     d * sumi - dmin * summ combine of :295-350, d * sumi of :352-386) in f32; the 4 threads
//     of a row add their partials, then the warps that split the row's superblocks add
//     theirs in a fixed order (deterministic, no atomics on data).
// The per-thread integer pieces add up exactly to the reference's sumi / summ; only the f32
// grouping differs (per thread share instead of per superblock), as in the lane GEMV.
//
// Shared memory: the stage row layout is chosen per context (KqParams::congruent): rows at
// their source's address mod 128 (whole-line bulk copies; a tile of whole rows is one copy)
// or at a row stride = 16 (mod 128), which puts the 16-byte loads of a warp's 8 rows in
// distinct banks. Q6_K superblocks (210 B) are only 2-byte aligned: a thread reads its 16
// bytes as 4 words in an order rotated by c (word (i + c) % 4 into slot i), which spreads
// those loads over the banks; the activations use the same rotation, so A and B agree.
//
// Pipeline: warp 16 is the producer (1-D bulk copies into a ring of stages, completion on
// mbarriers, L2 evict-first); warps 0..15 consume. A tile is 16 x rb rows of one job, split
// along k into slices of sl superblocks (one stage each); the warps of a 16-row block split
// a slice's superblocks. At the end of a tile every warp publishes its row partials to a
// shared buffer and the last warp to arrive (atomic counter, no barrier) adds and stores
// them. Every wait is bounded (2 s) and reports through the context's error word.
#include <algorithm>
#include <atomic>

#include "rcu_blocks.cuh"
#include "rcu_kernels.h"

namespace rcu {
namespace {

constexpr int kQW = 16;  // consumer warps
constexpr int kQThreads = (kQW + 1) * 32;
constexpr int kQMaxJobs = 96;
constexpr int kQMaxStages = 8;
constexpr int kQRed = 8;  // tile reduction buffers; must be >= the number of stages
constexpr uint32_t kQMaxStage = 64 * 1024;
constexpr int kQMaxPeers = 8;
constexpr uint32_t kQMaxStageRows = 64;

struct KqJob {
    const uint8_t *w;
    float *out;
    const uint32_t *sel;  // indirect (expert) job: weight = w + (*sel) * w_stride
    uint64_t w_stride;
    uint32_t rows, row_bytes, type, tok;
    uint32_t rb;           // 16-row blocks per tile
    uint32_t sl;           // superblocks per slice (one pipeline stage)
    uint32_t nsl;          // slices per tile
    uint32_t slice_bytes;  // sl * block bytes (a multiple of 16)
    uint32_t pstride;      // shared-memory row stride (see KqParams::congruent)
    uint32_t tile_begin;
};

struct KqParams {
    KqJob jobs[kQMaxJobs];
    int32_t n_jobs;
    uint32_t total_tiles, stages, stage_bytes, stage_off;
    uint32_t k, nsb, tok0, n_stage, early_weights;
    // Row layout in a stage. congruent: every row lands at the same address mod 128 as its
    // source (stage start shifted by the source's offset mod 128, row stride = row bytes mod
    // 128), so the bulk copies move whole 128-byte lines; a tile of whole contiguous rows is
    // one copy. Otherwise: row stride = 16 (mod 128), which spreads the 8 rows a warp reads
    // over all banks, at the price of copies whose source and destination lines differ.
    uint32_t congruent;
    uint32_t o_q, o_d, o_bs;  // shared-memory offsets of the staged Q8_K activations
    ActsView acts;
    uint32_t *err;
    // fused all-reduce push (as in rcu_gemv.cu); left zero by the launcher: launches that push
    // an all-reduce take the lane GEMV
    float *ar_dst[kQMaxPeers];
    uint32_t *ar_flag[kQMaxPeers];
    uint32_t ar_ndst, ar_nflag;
};

struct KqHdr {
    uint64_t full[kQMaxStages];
    uint64_t empty[kQMaxStages];
    int cnt[kQRed];
    float red[kQRed][kQW][16];  // [tile % kQRed][warp][row in the warp's 16-row block]
};
constexpr uint32_t kQHdrBytes = 8448;
static_assert(sizeof(KqHdr) <= kQHdrBytes, "header too large");
static_assert(kQRed >= kQMaxStages, "a warp can run up to (stages - 1) tiles ahead");

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
__device__ __forceinline__ void words8(const uint4 &x, const uint4 &y, uint32_t (&w)[8]) {
    w[0] = x.x, w[1] = x.y, w[2] = x.z, w[3] = x.w, w[4] = y.x, w[5] = y.y, w[6] = y.z, w[7] = y.w;
}

// Q4_K / Q5_K superblock at byte `so` of rows ra (row g) and rb (row g + 8); act: its 256
// activation codes, bsw: its 8 bsums pair words, ad: its activation scale.
template <int TYPE>
__device__ __forceinline__ void kq_q45(const uint8_t *ra, const uint8_t *rb, uint32_t so, const int8_t *act,
                                       const uint32_t *bsw, float ad, uint32_t c, bool bact, float &accA,
                                       float &accB) {
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
    uint32_t AL[8], AH[8];  // chunk c's activations: sub-block 2c (low) and 2c + 1 (high)
    if (bact) {
        const uint8_t *x = reinterpret_cast<const uint8_t *>(act) + 64 * c;
        words8(lds128(x), lds128(x + 16), AL);
        words8(lds128(x + 32), lds128(x + 48), AH);
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) AL[i] = AH[i] = 0u;
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
        mma_u8s8(dl, lo[0], lo[1], lo[2], lo[3], AL[2 * t], AL[2 * t + 1]);
        mma_u8s8(dh, hi[0], hi[1], hi[2], hi[3], AH[2 * t], AH[2 * t + 1]);
    }
    // scales of sub-blocks 2c, 2c + 1 and their mins (get_scale_min_k4, reference.rs:8-14)
    const uint2 bp = *reinterpret_cast<const uint2 *>(bsw + 2 * c);
    const uint32_t sh = 16u * (c & 1u);
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const uint4 hd = lds128(r ? pb : pa);
        const uint32_t a = hd.y >> sh, b = hd.w >> sh, cc = hd.z >> sh;
        const uint32_t scp = c < 2 ? a : ((b & 0x0F0Fu) | ((a >> 2) & 0x3030u));
        const uint32_t mnp = c < 2 ? cc : (((b >> 4) & 0x0F0Fu) | ((cc >> 2) & 0x3030u));
        const int s_lo = dl[2 * r], s_hi = TYPE == T_Q4_K ? (dh[2 * r] >> 4) : dh[2 * r];
        const int I = (int)(scp & 63u) * s_lo + (int)((scp >> 8) & 63u) * s_hi;
        const int M = dp2a_lo(bp.x, (mnp & 63u) * 0x0101u, dp2a_lo(bp.y, ((mnp >> 8) & 63u) * 0x0101u, 0));
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hd.x));
        float &acc = r ? accB : accA;
        acc = fmaf(ad, fmaf(-f.y, (float)M, f.x * (float)I), acc);
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
// superblock index).
template <bool A4>
__device__ __forceinline__ void kq_q6(const uint8_t *ra, const uint8_t *rb, uint32_t so, const int8_t *act,
                                      const uint32_t *bsw, float ad, uint32_t c, bool bact, float &accA,
                                      float &accB) {
    const uint32_t n = c >> 1, h = c & 1u;
    uint32_t LA0[4], LA1[4], HA[4], LB0[4], LB1[4], HB[4];
    ld4_rot<A4>(ra, so + 64 * n + 16 * h, c, LA0);
    ld4_rot<A4>(ra, so + 64 * n + 32 + 16 * h, c, LA1);
    ld4_rot<A4>(ra, so + 128 + 32 * n + 16 * h, c, HA);
    ld4_rot<A4>(rb, so + 64 * n + 16 * h, c, LB0);
    ld4_rot<A4>(rb, so + 64 * n + 32 + 16 * h, c, LB1);
    ld4_rot<A4>(rb, so + 128 + 32 * n + 16 * h, c, HB);
    uint32_t X[4][4];  // group (n, m, h) activations, rotated like the weights
    const uint8_t *xa = reinterpret_cast<const uint8_t *>(act) + 128 * n + 16 * h;
#pragma unroll
    for (int m = 0; m < 4; m++)
#pragma unroll
        for (int i = 0; i < 4; i++)
            X[m][i] = bact ? *reinterpret_cast<const uint32_t *>(xa + 32 * m + 4u * ((i + c) & 3u)) : 0u;
    int D[4][4];
#pragma unroll
    for (int m = 0; m < 4; m++) D[m][0] = D[m][1] = D[m][2] = D[m][3] = 0;
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const int i0 = 2 * u, i1 = 2 * u + 1;
        mma_u8s8(D[0], q6v<0>(LA0[i0], LA1[i0], HA[i0]), q6v<0>(LB0[i0], LB1[i0], HB[i0]),
                 q6v<0>(LA0[i1], LA1[i1], HA[i1]), q6v<0>(LB0[i1], LB1[i1], HB[i1]), X[0][i0], X[0][i1]);
        mma_u8s8(D[1], q6v<1>(LA0[i0], LA1[i0], HA[i0]), q6v<1>(LB0[i0], LB1[i0], HB[i0]),
                 q6v<1>(LA0[i1], LA1[i1], HA[i1]), q6v<1>(LB0[i1], LB1[i1], HB[i1]), X[1][i0], X[1][i1]);
        mma_u8s8(D[2], q6v<2>(LA0[i0], LA1[i0], HA[i0]), q6v<2>(LB0[i0], LB1[i0], HB[i0]),
                 q6v<2>(LA0[i1], LA1[i1], HA[i1]), q6v<2>(LB0[i1], LB1[i1], HB[i1]), X[2][i0], X[2][i1]);
        mma_u8s8(D[3], q6v<3>(LA0[i0], LA1[i0], HA[i0]), q6v<3>(LB0[i0], LB1[i0], HB[i0]),
                 q6v<3>(LA0[i1], LA1[i1], HA[i1]), q6v<3>(LB0[i1], LB1[i1], HB[i1]), X[3][i0], X[3][i1]);
    }
    // q6 - 32: subtract 32 x the group's activation sum (Q8_K bsums are per 16 values, one
    // per Q6_K scale group); groups 8n + 2m + h are the halves h of pair words 4n + m
    const uint4 bq = *reinterpret_cast<const uint4 *>(bsw + 4 * n);
    const uint32_t bw[4] = {bq.x, bq.y, bq.z, bq.w};
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
        acc = fmaf(f16_bits_to_f32(db) * ad, (float)I, acc);
    }
}

// One slice (sl superblocks starting at superblock sb0) of a warp's 16-row block: the
// warp takes superblocks part, part + wpb, ...
template <int TYPE>
__device__ __forceinline__ void kq_slice(const uint8_t *ra, const uint8_t *rb, uint32_t part, uint32_t wpb, uint32_t sl,
                                         uint32_t sb0, const int8_t *aq, const float *adk, const uint32_t *abw,
                                         uint32_t c, bool bact, float &accA, float &accB) {
    constexpr uint32_t BB = TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : 210;
    for (uint32_t sbl = part; sbl < sl; sbl += wpb) {
        const uint32_t sb = sb0 + sbl;
        const int8_t *act = aq + (size_t)sb * QK_K;
        const uint32_t *bsw = abw + 8 * sb;
        if (TYPE == T_Q6_K) {
            if (sbl & 1u)
                kq_q6<false>(ra, rb, sbl * BB, act, bsw, adk[sb], c, bact, accA, accB);
            else
                kq_q6<true>(ra, rb, sbl * BB, act, bsw, adk[sb], c, bact, accA, accB);
        } else {
            kq_q45<TYPE>(ra, rb, sbl * BB, act, bsw, adk[sb], c, bact, accA, accB);
        }
    }
}

// Destination shift of a stage whose source starts at `src` (congruent layout: the source's
// offset mod 128, a multiple of 16).
__device__ __forceinline__ uint32_t kq_shift(const KqParams &p, const uint8_t *src) {
    return p.congruent ? (uint32_t)(reinterpret_cast<uintptr_t>(src) & 127u) : 0u;
}

__device__ __forceinline__ void kq_store(const KqParams &p, const KqJob &jb, uint32_t row, float v) {
    jb.out[row] = v;
    for (uint32_t q = 0; q < p.ar_ndst; q++) p.ar_dst[q][row] = v;
}

__global__ void __launch_bounds__(kQThreads, 1) k_gemv_kq(const __grid_constant__ KqParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    KqHdr *h = reinterpret_cast<KqHdr *>(smem);
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

    if (warp == kQW) {  // ---- producer: one bulk copy per weight row and slice ----
        if (!p.early_weights) pdl_wait();
        const uint64_t pol = policy_evict_first();
        uint32_t li = 0, s = 0, ph = 0;  // stages issued, ring slot, pass parity
        int ji = 0;
        bool ok = true;
        for (uint32_t tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x) {
            while (ji + 1 < p.n_jobs && p.jobs[ji + 1].tile_begin <= tile) ji++;
            const KqJob &jb = p.jobs[ji];
            const uint32_t trows = 16u * jb.rb, r0 = (tile - jb.tile_begin) * trows;
            const uint32_t nrows = min(trows, jb.rows - r0);
            const uint32_t ex = jb.sel ? *jb.sel : 0u;
            for (uint32_t sl = 0; sl < jb.nsl; sl++) {
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
                    const uint8_t *src = jb.w + (uint64_t)ex * jb.w_stride + (uint64_t)r0 * jb.row_bytes +
                                         (uint64_t)sl * jb.slice_bytes;
                    uint8_t *dst = smem + p.stage_off + s * p.stage_bytes + kq_shift(p, src);
                    if (lane == 0) mbar_arrive_expect_tx(&h->full[s], nrows * jb.slice_bytes);
                    __syncwarp();
                    if (jb.nsl == 1 && jb.pstride == jb.row_bytes) {  // whole contiguous rows: one copy
                        if (lane == 0) bulk_g2s(dst, src, nrows * jb.row_bytes, &h->full[s], pol);
                    } else {
                        for (uint32_t r = lane; r < nrows; r += 32)
                            bulk_g2s(dst + r * jb.pstride, src + (uint64_t)r * jb.row_bytes, jb.slice_bytes,
                                     &h->full[s], pol);
                    }
                }
                li++;
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
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

    // ---- consumers: stage this call's Q8_K activations (rows tok0 .. tok0 + n_stage) ----
    pdl_wait();
    {
        const uint32_t nt = p.n_stage, k = p.k, nsb = p.nsb, tid = threadIdx.x, nthr = kQW * 32;
        const ActsView &A = p.acts;
        const uint4 *src = reinterpret_cast<const uint4 *>(A.qk + (size_t)p.tok0 * k);
        uint4 *dst = reinterpret_cast<uint4 *>(smem + p.o_q);
        for (uint32_t i = tid; i < nt * k / 16; i += nthr) dst[i] = src[i];
        for (uint32_t i = tid; i < nt * nsb; i += nthr)
            reinterpret_cast<float *>(smem + p.o_d)[i] = A.dk[(size_t)p.tok0 * nsb + i];
        const uint32_t *bsrc = reinterpret_cast<const uint32_t *>(A.bsk + (size_t)p.tok0 * (k / 16));
        for (uint32_t i = tid; i < nt * k / 32; i += nthr) reinterpret_cast<uint32_t *>(smem + p.o_bs)[i] = bsrc[i];
        named_bar_sync(1, nthr);
    }

    const uint32_t g = lane >> 2, c = lane & 3;
    const bool bact = c == (g >> 1);
    uint32_t s = 0, ph = 0, tloc = 0;
    int ji = 0;
    bool ok = true;
    for (uint32_t tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x, tloc++) {
        while (ji + 1 < p.n_jobs && p.jobs[ji + 1].tile_begin <= tile) ji++;
        const KqJob &jb = p.jobs[ji];
        const uint32_t trows = 16u * jb.rb, r0 = (tile - jb.tile_begin) * trows;
        const uint32_t nrows = min(trows, jb.rows - r0);
        const uint32_t ex = jb.sel ? *jb.sel : 0u;
        const bool skip = ex == kNoExpert;
        // stage shift of slice sl: (tile source + sl * slice bytes) mod 128, as the producer has it
        const uint32_t sh0 = kq_shift(p, jb.w + (uint64_t)(skip ? 0u : ex) * jb.w_stride + (uint64_t)r0 * jb.row_bytes);
        const uint32_t wpb = kQW / jb.rb, rbk = warp / wpb, part = warp % wpb;
        const int8_t *aq = reinterpret_cast<const int8_t *>(smem + p.o_q) + (size_t)jb.tok * p.k;
        const float *adk = reinterpret_cast<const float *>(smem + p.o_d) + (size_t)jb.tok * p.nsb;
        const uint32_t *abw = reinterpret_cast<const uint32_t *>(smem + p.o_bs) + (size_t)jb.tok * (p.k / 32);
        float accA = 0.0f, accB = 0.0f;
        for (uint32_t sl = 0; sl < jb.nsl; sl++) {
            if (!mbar_wait_bounded(&h->full[s], ph, p.err, ERR_TIMEOUT_FULL)) {
                ok = false;
                break;
            }
            if (!skip) {
                const uint32_t shift = p.congruent ? (sh0 + sl * jb.slice_bytes) & 127u : 0u;
                const uint8_t *ra = smem + p.stage_off + s * p.stage_bytes + shift + (rbk * 16u + g) * jb.pstride;
                const uint8_t *rb = ra + 8u * jb.pstride;
                const uint32_t sb0 = sl * jb.sl;
                switch (jb.type) {
                    case T_Q4_K: kq_slice<T_Q4_K>(ra, rb, part, wpb, jb.sl, sb0, aq, adk, abw, c, bact, accA, accB); break;
                    case T_Q5_K: kq_slice<T_Q5_K>(ra, rb, part, wpb, jb.sl, sb0, aq, adk, abw, c, bact, accA, accB); break;
                    default: kq_slice<T_Q6_K>(ra, rb, part, wpb, jb.sl, sb0, aq, adk, abw, c, bact, accA, accB); break;
                }
            }
            __syncwarp();
            if (sl + 1 == jb.nsl) {
                // tile done: the 4 threads of each row add their shares, every warp publishes
                // its rows' partials; the last warp to arrive adds the parts in order and stores
                accA += __shfl_xor_sync(0xffffffffu, accA, 1);
                accA += __shfl_xor_sync(0xffffffffu, accA, 2);
                accB += __shfl_xor_sync(0xffffffffu, accB, 1);
                accB += __shfl_xor_sync(0xffffffffu, accB, 2);
                const uint32_t ri = tloc % kQRed;
                if (c == 0) {
                    h->red[ri][warp][g] = accA;
                    h->red[ri][warp][g + 8] = accB;
                }
                __syncwarp();
                __threadfence_block();
                int old = 0;
                if (lane == 0) old = atomicAdd(&h->cnt[ri], 1);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == kQW - 1) {
                    __threadfence_block();
                    if (!skip) {
                        for (uint32_t i = lane; i < nrows; i += 32) {
                            const uint32_t bk = i >> 4, rr = i & 15u;
                            float v = 0.0f;
                            for (uint32_t q = 0; q < wpb; q++) v += *((volatile float *)&h->red[ri][bk * wpb + q][rr]);
                            kq_store(p, jb, r0 + i, v);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) atomicExch(&h->cnt[ri], 0);
                }
                __syncwarp();
            }
            if (lane == 0) mbar_arrive(&h->empty[s]);
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
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
// multiple of 8 superblocks so that 210-byte rows stay 16-byte multiples), 16-row blocks
// per tile rb (so that the 16 / rb warps of a block have a superblock each), stage bytes
// <= 64 KB. Prefers slices the block's warps split evenly, then longer slices.
bool kq_plan(const rcu_weight *w, uint32_t k, bool congruent, KqJob &jd) {
    const int t = w->type;
    if (t != T_Q4_K && t != T_Q5_K && t != T_Q6_K) return false;
    if (w->cols != k || k % QK_K != 0 || w->row_bytes % 16 != 0 || ((uintptr_t)w->data & 15u)) return false;
    const uint32_t bb = (uint32_t)block_bytes(t), nsb = k / QK_K;
    double best = -1.0;
    for (uint32_t sl = nsb; sl >= 1; sl--) {
        if (nsb % sl || (sl * bb) % 16) continue;
        uint32_t ps = sl * bb;
        if (congruent)
            ps += ((uint32_t)w->row_bytes - ps) % 128u;
        else
            ps += (16u + 128u - ps % 128u) % 128u;
        uint32_t rb = 1;
        while (kQW / rb > sl && rb < (uint32_t)kQW) rb *= 2;
        if (16u * rb * ps + (congruent ? 128u : 0u) > kQMaxStage) continue;
        const uint32_t wpb = kQW / rb;
        const double bal = (double)sl / (double)(wpb * ((sl + wpb - 1) / wpb));
        const double score = bal * 4.0 + (double)sl / nsb;
        if (score > best) {
            best = score;
            jd.sl = sl;
            jd.rb = rb;
            jd.pstride = ps;
        }
    }
    if (best < 0.0) return false;
    jd.nsl = nsb / jd.sl;
    jd.slice_bytes = jd.sl * bb;
    jd.type = (uint32_t)t;
    jd.row_bytes = (uint32_t)w->row_bytes;
    return true;
}

// Shared-memory layout of a launch: header, the staged Q8_K rows (codes, scales, bsums), then
// the weight stages. Returns false when two stages do not fit next to the staged rows.
bool kq_smem_layout(const rcu_ctx *ctx, uint32_t k, uint32_t n_rows, uint32_t stage_bytes, KqParams &p) {
    uint32_t off = kQHdrBytes;
    p.o_q = off;
    off = round_up_u(off + n_rows * k, 16);
    p.o_d = off;
    off = round_up_u(off + n_rows * (k / QK_K) * 4, 16);
    p.o_bs = off;
    off = round_up_u(off + n_rows * (k / 16) * 2, 16);
    p.stage_off = round_up_u(off, 128);
    const uint32_t budget = (uint32_t)ctx->max_smem_optin;
    if (p.stage_off + 2 * stage_bytes > budget) return false;
    p.stages = std::min<uint32_t>(kQMaxStages, (budget - p.stage_off) / stage_bytes);
    return true;
}

uint32_t kq_stage_bytes(const KqJob &jd, bool congruent) {
    return round_up_u(16 * jd.rb * jd.pstride + (congruent ? 128u : 0u), 128);
}

}  // namespace

bool gemv_kq_ok(const rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs) {
    if (!ctx->gemv_kq || n_jobs < 1 || n_jobs > kQMaxJobs || !(a.have & RCU_ACT_Q8K)) return false;
    uint64_t bytes = 0;
    uint32_t n_rows = 0, stage_bytes = 0;
    for (int i = 0; i < n_jobs; i++) {
        KqJob jd{};
        if (!kq_plan(jobs[i].w, a.k, ctx->gemv_kq_congruent, jd)) return false;
        if (jobs[i].sel && jobs[i].w_stride % 16 != 0) return false;
        if (jobs[i].tok + 1 > kQMaxStageRows) return false;
        bytes += (uint64_t)(jobs[i].rows ? jobs[i].rows : jobs[i].w->rows) * jobs[i].w->row_bytes;
        n_rows = std::max(n_rows, jobs[i].tok + 1);
        stage_bytes = std::max(stage_bytes, kq_stage_bytes(jd, ctx->gemv_kq_congruent));
    }
    KqParams lay;
    if (!kq_smem_layout(ctx, a.k, n_rows, stage_bytes, lay)) return false;
    // Small launches take the lane GEMV: this kernel's start-up (activation staging, the first
    // tile's latency chain) is longer, and with 1-2 tiles per CTA nothing hides it; K = 768
    // expert rows also give it few tiles (256-row tiles). Measured on B200: back-to-back launches
    // of one shape, 7 MB Q4_K 12.4 us here vs 6.0 lane, 9.4 MB 12.6 vs 8.1, 28 MB 12.5 vs 17.0,
    // 41 MB Q6_K 13.0 vs 21.5, 510 MB Q6_K 131 vs 260; serialized (profiler) 9.4 MB Q4_K 9.4 vs
    // 10.4 us, and the Qwen3-8B decode step (every launch >= 9.4 MB here) 2.67 ms vs 3.48 ms.
    return bytes >= ctx->gemv_kq_min_bytes;
}

int launch_gemv_kq(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs, uint32_t tok0) {
    KqParams p{};
    p.n_jobs = n_jobs;
    p.k = a.k;
    p.nsb = a.k / QK_K;
    p.tok0 = tok0;
    p.acts = a;
    p.err = ctx->dev_err;
    p.early_weights = ctx->early_weights ? 1u : 0u;
    p.congruent = ctx->gemv_kq_congruent ? 1u : 0u;
    uint32_t tiles = 0, stage_bytes = 0;
    for (int i = 0; i < n_jobs; i++) {
        KqJob &jd = p.jobs[i];
        if (!kq_plan(jobs[i].w, a.k, ctx->gemv_kq_congruent, jd))
            return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemv: weight not K-quant tileable");
        jd.w = jobs[i].w->data;
        jd.out = jobs[i].out + (jobs[i].sel ? 0 : (uint64_t)tok0 * jobs[i].ld);  // indirect jobs: own rows
        jd.sel = jobs[i].sel;
        jd.w_stride = jobs[i].w_stride;
        jd.tok = jobs[i].tok;
        jd.rows = jobs[i].rows ? jobs[i].rows : (uint32_t)jobs[i].w->rows;
        if (jd.sel) p.early_weights = 0;  // the producer reads the router's choice: wait first
        p.n_stage = std::max(p.n_stage, jd.tok + 1);
        jd.tile_begin = tiles;
        tiles += (jd.rows + 16 * jd.rb - 1) / (16 * jd.rb);
        stage_bytes = std::max(stage_bytes, kq_stage_bytes(jd, p.congruent != 0));
    }
    p.total_tiles = tiles;
    p.stage_bytes = stage_bytes;
    if (!kq_smem_layout(ctx, a.k, p.n_stage, stage_bytes, p))
        return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemv: activation rows + two weight stages exceed shared memory");
    const uint32_t smem_bytes = p.stage_off + p.stages * stage_bytes;
    const uint32_t grid = std::min<uint32_t>(tiles, (uint32_t)ctx->num_sms);
    static std::atomic<bool> attr_set[64] = {};  // per device; contexts may live on several threads
    if (!attr_set[ctx->device & 63].load(std::memory_order_acquire)) {
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_gemv_kq, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)ctx->max_smem_optin));
        attr_set[ctx->device & 63].store(true, std::memory_order_release);
    }
    RCU_CUDA_TRY(ctx, launch_k(ctx, k_gemv_kq, dim3(grid), dim3(kQThreads), smem_bytes, p));
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

}  // namespace rcu
