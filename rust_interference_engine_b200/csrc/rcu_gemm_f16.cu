// rcu_gemm_f16.cu -- prefill GEMM (n_tok >= kF16MinTok) for every GGUF weight type on the
// 5th-generation tensor cores, weights dequantized to f16 in shared memory.
//
//   Y[t][n] = sum_k W[n][k] * A[t][k]
//
// W[n][k] is the reference's dequantized weight (crates/rie-core/src/quant/reference.rs:53-215:
// d*(q-8), d*q+m, d*(q-16), d*q+m, d*q, d*sc*q - dmin*m, d*sc*(q-32)), computed in f32 and
// rounded once to f16; A[t][k] = d_a * q_a is the activation after the reference's Q8_0 / Q8_K
// quantization (quant/mod.rs:175-218), rounded once to f16 by k_acts_f16. The tensor core
// multiplies f16 x f16 exactly and accumulates in f32 over all of K, so the result differs from
// the reference's per-block integer sums (reference.rs:221-386, combined in f32) only by those
// two roundings, each at most 2^-11 relative per operand. One epilogue per output tile; the
// int8 kernel (rcu_gemm.cu) keeps exact per-block sums for Q4_0 and pays a per-block epilogue.
//
// Per CTA: a 128-weight-row x NT-token output tile (NT = 64, 128, 192 or 256) over all of K.
//   * warp 0    TMA producer: raw GGUF bytes, 256 values of K per row per raw stage (2-D tensor
//               map over [rows][row_bytes] in 16-bit elements), and f16 activation tiles of K 64
//               (128B-swizzled, K-major) per operand stage;
//   * warp 1    TMEM owner and MMA issuer: 4 x tcgen05.mma.kind::f16 (M = 128, N = NT, K = 16)
//               per operand stage, weights (A) read from tensor memory, activations (B) from
//               shared memory, into one f32 accumulator of NT TMEM columns;
//   * warps 2-17 dequantize: four threads per weight row, 16 values each per operand stage,
//               stored as packed f16 pairs into the stage's TMEM columns (tcgen05.st, lane =
//               weight row), which keeps the weight operand off the shared-memory port; after
//               the last stage the same warps read the accumulator (tcgen05.ld) and store Y.
// Up to kF16MaxJobs weights sharing the activations (q/k/v, gate/up) run in one launch: the
// grid's x dimension walks the row tiles of each job in turn.
// All waits are bounded; TMEM is freed on every exit path.
#include <cuda.h>

#include <algorithm>
#include <type_traits>

#include "rcu_blocks.cuh"
#include "rcu_kernels.h"
#include "rcu_tc.cuh"

namespace rcu {

constexpr int kHRows = 128;        // weight rows per CTA (MMA M)
constexpr int kHMaxTok = 256;      // tokens per CTA at most (MMA N)
constexpr int kHStages = 4;        // operand stages (K 64 each)
constexpr int kHAccCols = 256;     // TMEM columns of the f32 accumulator (one per token)
constexpr int kHTmemCols = 512;    // accumulator + kHStages weight stages of 32 columns
constexpr int kHRawStages = 2;     // raw GGUF stages (K 256 each)
constexpr int kHRawMax = 272;      // raw bytes per row per stage at most (Q8_0: 8 x 34)
constexpr int kHUnpackWarps = 16;  // 4 threads per weight row, 16 values each per stage
constexpr int kHThreads = (2 + kHUnpackWarps) * 32;
constexpr int kF16MaxJobs = 4;
constexpr int kGrpMaxItems = 512;    // grouped (per-expert) launches: (expert, token tile) items
constexpr int kGrpMaxExperts = 256;
constexpr uint32_t kF16MinTok = 32;  // below this the 8-token GEMV slices are used

struct HSmem {
    uint8_t b[kHStages][kHMaxTok * 128];    // f16 activations (TMA, 128B swizzle)
    uint8_t raw[kHRawStages][kHRows * kHRawMax];
    uint64_t raw_full[kHRawStages], raw_empty[kHRawStages];
    uint64_t b_full[kHStages], a_full[kHStages], ab_empty[kHStages];
    uint64_t acc_full;
    uint32_t tmem_base;
};

struct HJob {
    float *out;
    uint64_t ld;
    uint32_t rows, tile0;  // weight rows; first grid-x tile of this job
};
struct HMaps {
    CUtensorMap w[kF16MaxJobs];
};
struct HParams {
    HJob job[kF16MaxJobs];
    const float *tok_scale;  // [n_tok] power of two that undoes the activation row's f16 scaling
    uint32_t n_jobs, k, n_tok, nt, idesc;
    int early;  // weights may be loaded before the grid dependency wait
    uint32_t *err;
    // grouped mode (grp > 0, mixture of experts): each job is a stacked expert tensor of
    // grp_rows rows per expert; blockIdx.y is work item i = (expert grp_exp[i], token tile
    // grp_tile[i]) over the activation rows [grp_off[e], grp_off[e + 1]) of that expert, and
    // blockIdx.x - tile0 the row tile within the expert. Output row = activation row.
    uint32_t grp, grp_rows;
    // split K (one job, plain mode): blockIdx.z takes units [z * nu / splits, (z + 1) * nu /
    // splits) of the nu = k / 256; every split writes its scaled tile to part[z] ([n_tok][rows]),
    // and the last CTA of the output tile (counter cnt[tile], reset by it) adds them in z order
    uint32_t splits;
    float *part;
    uint32_t *cnt;
    uint16_t grp_exp[kGrpMaxItems], grp_tile[kGrpMaxItems];
    uint32_t grp_off[kGrpMaxExperts + 1];
};

// ---- dequantization of 32 values of one row -----------------------------------------------
template <int TYPE>
constexpr uint32_t unit_bytes_c() {  // bytes of 256 values of K
    return TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : TYPE == T_Q6_K ? 210 : 8 * blk_bytes_c<TYPE>();
}
// Raw stage box per row. Q6_K superblocks (210 B) start on even, not 16-byte, offsets, so its
// box starts at the 16-byte boundary below and is wide enough for any start within 16 bytes.
// Every box is an odd number of 16-byte chunks (Q4_1 and Q5_1 rows carry one spare chunk):
// 8 consecutive rows then start in 8 different bank groups, so the 16-byte reads of a warp's
// 8-lane phases are conflict-free.
template <int TYPE>
constexpr uint32_t raw_box_c() {
    return TYPE == T_Q6_K ? 240 : TYPE == T_Q4_1 ? 176 : TYPE == T_Q5_1 ? 208 : unit_bytes_c<TYPE>();
}
static_assert(raw_box_c<T_Q4_0>() % 32 == 16 && raw_box_c<T_Q4_1>() % 32 == 16 && raw_box_c<T_Q5_0>() % 32 == 16 &&
                  raw_box_c<T_Q5_1>() % 32 == 16 && raw_box_c<T_Q8_0>() % 32 == 16 &&
                  raw_box_c<T_Q4_K>() % 32 == 16 && raw_box_c<T_Q5_K>() % 32 == 16 && raw_box_c<T_Q6_K>() % 32 == 16,
              "raw rows must be an odd number of 16-byte chunks");

// ---- 16 values of one row as 8 packed f16 pairs ---------------------------------------------
// 32-value block types: each code byte becomes the f16 1024 + code (byte placed in the mantissa
// of 0x6400), one subtraction makes the code exact, one f16 multiply (or fma with the min) by the
// f16 block scale rounds once: the same value as the f32 product rounded to f16.
// K-quants: the code becomes the f32 2^23 + code, an f32x2 add makes it exact, an f32x2 fma with
// d*sc (exact in f32) and -dmin*m rounds once in f32, and the pair is rounded to f16.
__device__ __forceinline__ uint32_t h2_pair(uint32_t w, uint32_t sel) { return __byte_perm(w, 0x64646464u, sel); }
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, __half2 b) {
    const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&a), b);
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, __half2 b) {
    const __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&a), b);
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, __half2 b, __half2 c) {
    const __half2 r = __hfma2(*reinterpret_cast<const __half2 *>(&a), b, c);
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t h2u(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(*reinterpret_cast<uint64_t *>(&a)), "l"(*reinterpret_cast<uint64_t *>(&b)));
    return *reinterpret_cast<float2 *>(&r);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(r)
        : "l"(*reinterpret_cast<uint64_t *>(&a)), "l"(*reinterpret_cast<uint64_t *>(&b)),
          "l"(*reinterpret_cast<uint64_t *>(&c)));
    return *reinterpret_cast<float2 *>(&r);
}
// Bytes (e, e+1) of w (codes 0..255) as the f32 pair 2^23 + code.
__device__ __forceinline__ float2 magic2(uint32_t w, uint32_t e) {
    return make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | e)),
                       __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (e + 1))));
}

// 4 code words (16 codes, byte order = value order) -> 8 f16 pairs, w = (code - bias) * d [+ m].
template <bool MIN>
__device__ __forceinline__ void codes_f16(const uint32_t (&c)[4], float bias, float d, float m, uint32_t (&o)[8]) {
    const __half2 b2 = __float2half2_rn(1024.0f + bias), d2 = __float2half2_rn(d), m2 = __float2half2_rn(m);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t lo = h2_sub(h2_pair(c[i], 0x5140u), b2), hi = h2_sub(h2_pair(c[i], 0x7362u), b2);
        o[2 * i] = MIN ? h2_fma(lo, d2, m2) : h2_mul(lo, d2);
        o[2 * i + 1] = MIN ? h2_fma(hi, d2, m2) : h2_mul(hi, d2);
    }
}
// 4 code words -> 8 f16 pairs, w = fma(code - bias, ds, -dm) in f32 (K-quants).
__device__ __forceinline__ void codes_f32(const uint32_t (&c)[4], float bias, float ds, float dm, uint32_t (&o)[8]) {
    const float2 nb = make_float2(-8388608.0f - bias, -8388608.0f - bias), s2 = make_float2(ds, ds),
                 m2 = make_float2(-dm, -dm);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 a = fma2(add2(magic2(c[i], 0), nb), s2, m2), b = fma2(add2(magic2(c[i], 2), nb), s2, m2);
        o[2 * i] = h2u(a.x, a.y);
        o[2 * i + 1] = h2u(b.x, b.y);
    }
}

// N words starting at the even byte offset `off` of a 16-byte aligned shared-memory row, read as
// the 16-byte chunks around them. With `off` known at compile time the selects fold away.
template <int N>
__device__ __forceinline__ void ldw16(const uint8_t *row, uint32_t off, uint32_t (&out)[N]) {
    constexpr int M = (4 * N + 14 + 15) / 16;  // chunks covering any even start within a chunk
    static_assert(4 * M >= N + 4, "chunk window");
    const uint4 *p = reinterpret_cast<const uint4 *>(row + (off & ~15u));
    uint32_t r[4 * M];
#pragma unroll
    for (int m = 0; m < M; m++) {
        const uint4 v = p[m];
        r[4 * m] = v.x, r[4 * m + 1] = v.y, r[4 * m + 2] = v.z, r[4 * m + 3] = v.w;
    }
    const uint32_t k = (off >> 2) & 3u, sh = (off & 3u) * 8u;
    uint32_t t[N + 1];
#pragma unroll
    for (int i = 0; i <= N; i++) {
        const uint32_t a = (k & 2u) ? r[i + 2] : r[i], b = (k & 2u) ? r[i + 3] : r[i + 1];
        t[i] = (k & 1u) ? b : a;
    }
#pragma unroll
    for (int i = 0; i < N; i++) out[i] = __funnelshift_r(t[i], t[i + 1], sh);
}

// Values [32 J + 16 h, +16) of the 256-value unit that starts `ofs` bytes into `row` (a 16-byte
// aligned row of a raw stage), dequantized as reference.rs:53-207 defines them, as f16 pairs.
template <int TYPE, int J>
__device__ __forceinline__ void dq16(const uint8_t *row, uint32_t ofs, uint32_t h, uint32_t (&o)[8]) {
    uint32_t c[4];
    if constexpr (TYPE == T_Q4_0) {  // d, qs[16]: low nibbles = values 0..15, high = 16..31
        uint32_t w[5];
        ldw16<5>(row, J * 18, w);
#pragma unroll
        for (int i = 0; i < 4; i++) c[i] = (__funnelshift_r(w[i], w[i + 1], 16) >> (4 * h)) & 0x0F0F0F0Fu;
        codes_f16<false>(c, 8.0f, f16_bits_to_f32(w[0]), 0.0f, o);
    } else if constexpr (TYPE == T_Q8_0) {  // d, qs[32] int8
        uint32_t d[1];
        ldw16<1>(row, J * 34, d);
        ldw16<4>(row, J * 34 + 2 + 16 * h, c);
#pragma unroll
        for (int i = 0; i < 4; i++) c[i] ^= 0x80808080u;
        codes_f16<false>(c, 128.0f, f16_bits_to_f32(d[0]), 0.0f, o);
    } else if constexpr (TYPE == T_Q5_0) {  // d, qh (u32), qs[16]; bit l of qh is the 5th bit of value l
        uint32_t w[6];
        ldw16<6>(row, J * 22, w);
        const uint32_t qh = __funnelshift_r(w[0], w[1], 16);
#pragma unroll
        for (int i = 0; i < 4; i++)
            c[i] = ((__funnelshift_r(w[1 + i], w[2 + i], 16) >> (4 * h)) & 0x0F0F0F0Fu) |
                   spread4_bit4(qh >> (16 * h + 4 * i));
        codes_f16<false>(c, 16.0f, f16_bits_to_f32(w[0]), 0.0f, o);
    } else if constexpr (TYPE == T_Q4_1 || TYPE == T_Q5_1) {  // d, m, [qh], qs[16]
        constexpr int Q = TYPE == T_Q4_1 ? 1 : 2;
        uint32_t w[4 + Q];
        ldw16<4 + Q>(row, J * blk_bytes_c<TYPE>(), w);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            c[i] = (w[Q + i] >> (4 * h)) & 0x0F0F0F0Fu;
            if (TYPE == T_Q5_1) c[i] |= spread4_bit4(w[1] >> (16 * h + 4 * i));
        }
        codes_f16<true>(c, 0.0f, f16_bits_to_f32(w[0]), f16_bits_to_f32(w[0] >> 16), o);
    } else if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        // d, dmin, 12 scale bytes, [Q5_K: qh 32 B], qs 128 B (reference.rs:153-189); sub-block J
        const uint4 hd = *reinterpret_cast<const uint4 *>(row);
        // get_scale_min_k4 (reference.rs:8-14)
        constexpr uint32_t sh = 8 * (J & 3);
        const uint32_t b0 = (hd.y >> sh) & 0xffu, b1 = (hd.z >> sh) & 0xffu, b2 = (hd.w >> sh) & 0xffu;
        const uint32_t sc = J < 4 ? b0 & 63u : (b2 & 0xFu) | ((b0 >> 6) << 4);
        const uint32_t mn = J < 4 ? b1 & 63u : (b2 >> 4) | ((b1 >> 6) << 4);
        const float ds = f16_bits_to_f32(hd.x) * (float)sc, dm = f16_bits_to_f32(hd.x >> 16) * (float)mn;
        constexpr uint32_t qs_off = TYPE == T_Q4_K ? 16 : 48;
        const uint4 q = *reinterpret_cast<const uint4 *>(row + qs_off + 32 * (J >> 1) + 16 * h);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        uint4 hb = make_uint4(0, 0, 0, 0);
        if (TYPE == T_Q5_K) hb = *reinterpret_cast<const uint4 *>(row + 16 + 16 * h);  // qh[16h..16h+16)
        const uint32_t hw[4] = {hb.x, hb.y, hb.z, hb.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            c[i] = ((J & 1) ? qw[i] >> 4 : qw[i]) & 0x0F0F0F0Fu;
            if (TYPE == T_Q5_K) c[i] |= ((hw[i] >> J) & 0x01010101u) << 4;  // bit J of qh[l]
        }
        codes_f32(c, 0.0f, ds, dm, o);
    } else {  // Q6_K: ql 128 B, qh 64 B, 16 int8 scales, d (reference.rs:190-207); group J
        constexpr uint32_t n = J >> 2, jj = J & 3;
        uint32_t ql[4], qh[4], sd[5];
        ldw16<4>(row, ofs + 64 * n + 32 * (jj & 1) + 16 * h, ql);
        ldw16<4>(row, ofs + 128 + 32 * n + 16 * h, qh);
        ldw16<5>(row, ofs + 192, sd);  // scales[16], d
        const uint32_t si = 8 * n + 2 * jj;  // scale of values l < 16; l >= 16 uses si + 1
        const int sc = (int)(int8_t)(__funnelshift_r(sd[si >> 2], sd[(si >> 2) + 1], 8 * (si & 3) + 8 * h) & 0xffu);
        const float ds = f16_bits_to_f32(sd[4]) * (float)sc;
#pragma unroll
        for (int i = 0; i < 4; i++)
            c[i] = (jj < 2 ? ql[i] & 0x0F0F0F0Fu : (ql[i] >> 4) & 0x0F0F0F0Fu) |
                   (((qh[i] >> (2 * jj)) & 0x03030303u) << 4);
        codes_f32(c, 32.0f, ds, 0.0f, o);
    }
}

// D[tmem] (+)= A[tmem] * B[smem descriptor]^T: the weights come from tensor memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"((uint32_t)acc)
        : "memory");
}
// 8 columns of this warp's 32 TMEM lanes, one 32-bit register per column and thread.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// AND of v over the nthreads threads (whole warps) that reach named barrier id.
__device__ __forceinline__ bool bar_and(int id, int nthreads, bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n barrier.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// Every lane of the warp waits; the warp gives up together if any lane timed out.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, uint32_t *err, uint32_t code) {
    const bool ok = mbar_wait_bounded(bar, parity, err, code);
    return __all_sync(0xffffffffu, ok);
}

template <int TYPE>
__global__ void __launch_bounds__(kHThreads, 1)
    k_gemm_f16(const __grid_constant__ HMaps maps, const __grid_constant__ CUtensorMap map_b,
               const __grid_constant__ HParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    HSmem &S = *reinterpret_cast<HSmem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    constexpr uint32_t UB = unit_bytes_c<TYPE>(), BOX = raw_box_c<TYPE>();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t ji = 0;
    while (ji + 1 < p.n_jobs && blockIdx.x >= p.job[ji + 1].tile0) ji++;
    const HJob &jb = p.job[ji];
    // tile origin: weight row in the tensor map (wrow0), output column (col0, valid below
    // col_lim), first activation / output row (trow0) and its valid count (tcount)
    uint32_t wrow0, col0, col_lim, trow0, tcount;
    if (p.grp) {
        const uint32_t ex = p.grp_exp[blockIdx.y], t0 = p.grp_tile[blockIdx.y] * p.nt;
        col0 = (blockIdx.x - jb.tile0) * kHRows;
        wrow0 = ex * p.grp_rows + col0;
        col_lim = p.grp_rows;
        trow0 = p.grp_off[ex] + t0;
        tcount = p.grp_off[ex + 1] - p.grp_off[ex] - t0;
    } else {
        col0 = wrow0 = (blockIdx.x - jb.tile0) * kHRows;
        col_lim = jb.rows;
        trow0 = blockIdx.y * p.nt;
        tcount = p.n_tok - trow0;
    }
    const uint32_t nu_all = p.k / QK_K, u_beg = blockIdx.z * nu_all / p.splits;
    const uint32_t n_unit = (blockIdx.z + 1) * nu_all / p.splits - u_beg, n_it = n_unit * 4;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kHRawStages; s++) {
            mbar_init(&S.raw_full[s], 1);
            mbar_init(&S.raw_empty[s], kHUnpackWarps);
        }
        for (int s = 0; s < kHStages; s++) {
            mbar_init(&S.b_full[s], 1);
            mbar_init(&S.a_full[s], kHUnpackWarps);
            mbar_init(&S.ab_empty[s], 1);
        }
        mbar_init(&S.acc_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc<kHTmemCols>(&S.tmem_base);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;

    if (warp == 0) {  // ---- TMA producer ----
        if (lane == 0) {
            const CUtensorMap *mw = &maps.w[ji];
            uint32_t units = 0, its = 0;  // issued
            bool ok = true;
            auto issue_raw = [&](uint32_t u) -> bool {
                const uint32_t rs = u % kHRawStages;
                if (u >= kHRawStages &&
                    !mbar_wait_bounded(&S.raw_empty[rs], ((u / kHRawStages) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY))
                    return false;
                mbar_arrive_expect_tx(&S.raw_full[rs], BOX * kHRows);
                tma_load_2d(S.raw[rs], mw, (int)((((u_beg + u) * UB) & ~15u) >> 1), (int)wrow0, &S.raw_full[rs]);
                units = u + 1;
                return true;
            };
            if (p.early) issue_raw(0);  // weights are written once, before any forward
            pdl_wait();
            pdl_trigger();
            if (!p.early) ok = issue_raw(0);
            for (uint32_t it = 0; it < n_it && ok; it++) {
                if ((it & 3) == 0 && (it >> 2) + 1 < n_unit && !issue_raw((it >> 2) + 1)) ok = false;
                const uint32_t s = it % kHStages;
                if (!ok ||
                    (it >= kHStages && !mbar_wait_bounded(&S.ab_empty[s], ((it / kHStages) - 1) & 1, p.err,
                                                          ERR_TIMEOUT_EMPTY))) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&S.b_full[s], p.nt * 128);
                tma_load_2d(S.b[s], &map_b, (int)((u_beg * 4 + it) * 64), (int)trow0, &S.b_full[s]);
                its = it + 1;
            }
            // drain: the last copy issued into each stage has landed (already true unless a
            // consumer gave up), so no copy is in flight when the CTA exits
            for (uint32_t u = units > kHRawStages ? units - kHRawStages : 0; u < units; u++)
                mbar_wait_bounded(&S.raw_full[u % kHRawStages], (u / kHRawStages) & 1, p.err, ERR_TIMEOUT_DRAIN);
            for (uint32_t it = its > kHStages ? its - kHStages : 0; it < its; it++)
                mbar_wait_bounded(&S.b_full[it % kHStages], (it / kHStages) & 1, p.err, ERR_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {  // ---- MMA issuer ----
        if (lane == 0) {
            for (uint32_t it = 0; it < n_it; it++) {
                const uint32_t s = it % kHStages, ph = (it / kHStages) & 1;
                if (!mbar_wait_bounded(&S.b_full[s], ph, p.err, ERR_TIMEOUT_FULL) ||
                    !mbar_wait_bounded(&S.a_full[s], ph, p.err, ERR_TIMEOUT_FULL))
                    break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    mma_f16_ts(tmem, tmem + kHAccCols + 32 * s + 8 * kk, sw128_desc(S.b[s] + 32 * kk), p.idesc,
                               (it | kk) != 0);
                mma_commit(&S.ab_empty[s]);
            }
            mma_commit(&S.acc_full);  // also on an early exit: tracks every MMA issued
        }
    } else {  // ---- dequantize, then epilogue (warps 2-17) ----
        // a warp may only reach TMEM lanes 32 (warp % 4) .. +31: warp (q, part) dequantizes rows
        // 32 q .. 32 q + 31, values [16 part, +16) of every operand stage
        const uint32_t q = warp & 3, part = (warp - 2) >> 2, r = 32 * q + lane;
        static_assert(kHStages == 4, "one unit of K 256 = kHStages operand stages");
        const uint32_t rh = part & 1;  // which half of its 32-value group this thread dequantizes
        bool ok = true;
        for (uint32_t u = 0; u < n_unit && ok; u++) {
            const uint32_t rs = u % kHRawStages, ofs = ((u_beg + u) * UB) & 15u;
            if (!warp_wait(&S.raw_full[rs], (u / kHRawStages) & 1, p.err, ERR_TIMEOUT_FULL)) {
                ok = false;
                break;
            }
            const uint8_t *rrow = S.raw[rs] + r * BOX;
            // operand stage G of this unit (values [64 G, +64)); G is a compile-time constant so
            // that the 32-value group index and its byte offsets are too
            auto stage = [&](auto gc) -> bool {
                constexpr int G = decltype(gc)::value;
                if (u > 0 && !warp_wait(&S.ab_empty[G], (u - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) return false;
                tc_fence_after();  // the MMA that read this weight stage has completed
                uint32_t o[8];
                if (part >> 1)  // warp-uniform
                    dq16<TYPE, 2 * G + 1>(rrow, ofs, rh, o);
                else
                    dq16<TYPE, 2 * G>(rrow, ofs, rh, o);
                // K values [16 part, +16) of this stage: 8 columns of packed f16 pairs, lane = row
                tmem_st8(tmem + ((32 * q) << 16) + kHAccCols + 32 * G + 8 * part, o);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&S.a_full[G]);
                    if (G == 3) mbar_arrive(&S.raw_empty[rs]);
                }
                return true;
            };
            ok = stage(std::integral_constant<int, 0>{}) && stage(std::integral_constant<int, 1>{}) &&
                 stage(std::integral_constant<int, 2>{}) && stage(std::integral_constant<int, 3>{});
        }
        pdl_wait();  // the output may still be read by the kernel before this one
        bool acc_ok = ok && warp_wait(&S.acc_full, 0, p.err, ERR_TIMEOUT_FULL);
        // the epilogue warps agree, so that its named barriers see all of them or none
        acc_ok = bar_and(1, kHUnpackWarps * 32, acc_ok);
        if (acc_ok) {
            tc_fence_after();
            // the four warps of a lane quarter split the accumulator columns
            const uint32_t span = p.nt / (kHUnpackWarps / 4);
            const uint32_t n = col0 + r;
            // one split: the output; several: this split's slice of the partial sums
            float *dst = p.splits > 1 ? p.part + (uint64_t)blockIdx.z * p.n_tok * jb.rows : jb.out;
            const uint64_t ld = p.splits > 1 ? jb.rows : jb.ld;
            for (uint32_t c = part * span; c < (part + 1) * span; c += 16) {
                uint32_t x[16];
                tmem_ld16(tmem + ((32 * q) << 16) + c, x);
                tmem_wait_ld();
                if (n < col_lim) {
#pragma unroll
                    for (int e = 0; e < 16; e++) {
                        const uint32_t m = trow0 + c + e;
                        if (c + e < tcount) dst[(uint64_t)m * ld + n] = __uint_as_float(x[e]) * p.tok_scale[m];
                    }
                }
            }
            if (p.splits > 1) {  // the last split of this output tile adds the partial tiles in order
                __shared__ uint32_t s_last;
                __threadfence();
                named_bar_sync(1, kHUnpackWarps * 32);
                const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
                if (warp == 2 && lane == 0) {
                    const uint32_t done = atomicAdd(p.cnt + tile, 1u);
                    s_last = done == p.splits - 1;
                    if (s_last) p.cnt[tile] = 0;  // ready for the next launch
                }
                named_bar_sync(1, kHUnpackWarps * 32);
                if (s_last) {
                    // this split's values come from TMEM again, the others' from the partial
                    // tiles (16 independent loads in flight per split), summed in split order
                    __threadfence();
                    for (uint32_t c = part * span; c < (part + 1) * span; c += 16) {
                        uint32_t x[16];
                        tmem_ld16(tmem + ((32 * q) << 16) + c, x);
                        tmem_wait_ld();
                        if (n >= col_lim) continue;
                        float acc[16];
#pragma unroll
                        for (int e = 0; e < 16; e++) acc[e] = 0.0f;
                        for (uint32_t z = 0; z < p.splits; z++) {
                            float v[16];
#pragma unroll
                            for (int e = 0; e < 16; e++) {
                                const uint32_t m = trow0 + c + e;
                                v[e] = z == blockIdx.z ? __uint_as_float(x[e]) * p.tok_scale[m]
                                       : c + e < tcount ? __ldcg(p.part + ((uint64_t)z * p.n_tok + m) * jb.rows + n)
                                                        : 0.0f;
                            }
#pragma unroll
                            for (int e = 0; e < 16; e++) acc[e] += v[e];
                        }
#pragma unroll
                        for (int e = 0; e < 16; e++)
                            if (c + e < tcount) jb.out[(uint64_t)(trow0 + c + e) * jb.ld + n] = acc[e];
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        // every MMA has completed before the accumulator is released (immediate unless a
        // wait above gave up)
        if (lane == 0) mbar_wait_bounded(&S.acc_full, 0, p.err, ERR_TIMEOUT_DRAIN);
        __syncwarp();
        tc_fence_after();
        tmem_free<kHTmemCols>(tmem);
    }
}

// A[t][k] = f16(d_a * q_a * 2^-e_t) of the prepared Q8_0 or Q8_K activations, one CTA per token
// row. e_t >= 0 is the smallest power that keeps the row's largest value (127 * max |d_a|) within
// 2^15, so that no value overflows f16 (activations of some models reach 1e5); tok_scale[t] = 2^e_t
// is multiplied back, exactly, in the GEMM epilogue. Rows already in range are unchanged.
constexpr int kActsF16Threads = 256;
// src_rows != nullptr gathers: output row i is activation row src_rows[i] (grouped GEMM).
__global__ void __launch_bounds__(kActsF16Threads) k_acts_f16(const ActsView a, uint32_t fmt, __half *__restrict__ out,
                                                              float *__restrict__ tok_scale,
                                                              const uint32_t *__restrict__ src_rows) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[kActsF16Threads / 32];
    const uint32_t row = blockIdx.x, t = src_rows ? src_rows[row] : row, tid = threadIdx.x;
    const bool q0 = fmt == RCU_ACT_Q8_0;
    const uint32_t bs = q0 ? QK : QK_K, nb = a.k / bs;
    const float *dr = (q0 ? a.d0 : a.dk) + (uint64_t)t * nb;
    float mx = 0.0f;
    for (uint32_t b = tid; b < nb; b += kActsF16Threads) mx = fmaxf(mx, fabsf(dr[b]));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = 0.0f;
#pragma unroll
    for (int w = 0; w < kActsF16Threads / 32; w++) mx = fmaxf(mx, red[w]);
    // e = max(0, ceil(log2(127 * mx / 2^15))), from the exponent of the (finite) bound
    const float amax = 127.0f * mx;
    int e = 0;
    if (amax > 32768.0f) {
        const int ex = (int)((__float_as_uint(amax) >> 23) & 0xffu) - 127;  // amax in [2^ex, 2^(ex+1))
        e = ex - 14;                                                         // amax / 2^e < 2^15
    }
    const float down = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e (e <= 113 for finite input)
    if (tid == 0) tok_scale[row] = __uint_as_float((uint32_t)(127 + e) << 23);
    const int8_t *qs = (q0 ? a.q0 : a.qk) + (uint64_t)t * a.k;
    __half *orow = out + (uint64_t)row * a.k;
    for (uint32_t i = tid * 8; i < a.k; i += kActsF16Threads * 8) {
        const uint2 c = *reinterpret_cast<const uint2 *>(qs + i);
        const float d = dr[i / bs] * down;  // exact: a power-of-two scaling
        uint4 o;
        o.x = h2u((float)sbyte(c.x, 0) * d, (float)sbyte(c.x, 1) * d);
        o.y = h2u((float)sbyte(c.x, 2) * d, (float)sbyte(c.x, 3) * d);
        o.z = h2u((float)sbyte(c.y, 0) * d, (float)sbyte(c.y, 1) * d);
        o.w = h2u((float)sbyte(c.y, 2) * d, (float)sbyte(c.y, 3) * d);
        *reinterpret_cast<uint4 *>(orow + i) = o;
    }
}

// ---- host side -----------------------------------------------------------------------------
static bool f16_type_ok(int t) { return gemv_supported(t); }

bool gemm_f16_ok(const ActsView &a, const HostJob &j) {
    const rcu_weight *w = j.w;
    if (!f16_type_ok(w->type) || j.sel || j.tok) return false;
    if (a.k % QK_K != 0 || (w->row_bytes & 15) != 0 || (((uintptr_t)w->data) & 15) != 0) return false;
    if (w->rows >= (1ull << 31)) return false;
    return a.n_tok >= kF16MinTok;
}

// Tokens per CTA and K splits: the fewest waves of CTAs, a CTA costing about (nt + 64) per unit
// of K 256 plus two units of fixed cost (the dequantization of its weight tile is paid once per
// token tile). A single-weight launch may split K in 2 or 4 (at least 2 units per split,
// partial sums at most 64 MB), paying for the ordered reduction of the partials. Measured on
// 512 tokens: ffn_down 4096 x 12288 Q6_K 126 -> 88 us (2 splits), attn_v 1024 x 4096 Q6_K 45 ->
// 32 us (4); more splits than 4 were slower everywhere.
static void pick_tiling(uint64_t tiles_w, uint32_t n_tok, uint32_t n_unit, uint64_t split_rows, int sms, uint32_t *nt_out,
                        uint32_t *splits_out) {
    double best = 1e300;
    *nt_out = 64, *splits_out = 1;
    for (uint32_t nt : {256u, 192u, 128u, 64u})
        for (uint32_t sp : {1u, 2u, 4u}) {
            if (sp > 1 && (split_rows == 0 || n_unit / sp < 2 ||
                           (uint64_t)sp * n_tok * split_rows * 4 > (64ull << 20)))
                continue;
            const uint64_t ctas = tiles_w * ((n_tok + nt - 1) / nt) * sp;
            const double per = ((double)n_unit / sp + 2.0) * (nt + 64) + (sp > 1 ? sp * nt / 2.0 : 0.0);
            const double cost = (double)((ctas + sms - 1) / sms) * per;
            if (cost < best) best = cost, *nt_out = nt, *splits_out = sp;
        }
}

static int ensure_split_scratch(rcu_ctx *ctx, size_t part_bytes, size_t cnt_bytes) {
    if (ctx->k_part_cap < part_bytes) {
        RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        if (ctx->k_part) cudaFree(ctx->k_part);
        ctx->k_part = nullptr;
        ctx->k_part_cap = 0;
        RCU_CUDA_TRY(ctx, cudaMalloc(&ctx->k_part, part_bytes));
        ctx->k_part_cap = part_bytes;
    }
    if (ctx->k_cnt_cap < cnt_bytes) {  // counters start at zero; each launch leaves them at zero
        RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        if (ctx->k_cnt) cudaFree(ctx->k_cnt);
        ctx->k_cnt = nullptr;
        ctx->k_cnt_cap = 0;
        RCU_CUDA_TRY(ctx, cudaMalloc((void **)&ctx->k_cnt, cnt_bytes));
        RCU_CUDA_TRY(ctx, cudaMemset(ctx->k_cnt, 0, cnt_bytes));
        ctx->k_cnt_cap = cnt_bytes;
    }
    return RCU_OK;
}

static int ensure_f16_scratch(rcu_ctx *ctx, size_t bytes) {
    if (ctx->h_act_cap >= bytes) return RCU_OK;
    RCU_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->h_act) cudaFree(ctx->h_act);
    ctx->h_act = nullptr;
    ctx->h_act_cap = 0;
    if (cudaMalloc(&ctx->h_act, bytes) != cudaSuccess) {
        cudaGetLastError();
        ctx->h_act = nullptr;
        return set_err(ctx, RCU_ERR_OOM, "f16 activation scratch");
    }
    ctx->h_act_cap = bytes;
    return RCU_OK;
}

// f16 activations [n_tok][k], then the per-token scales [n_tok]
static size_t f16_scratch_bytes(uint64_t n_tok, uint64_t k) { return ((n_tok * k * 2 + 255) & ~(size_t)255) + n_tok * 4; }
int gemm_f16_reserve(rcu_ctx *ctx, uint64_t n_tok, uint64_t k) {
    return ensure_f16_scratch(ctx, f16_scratch_bytes(n_tok, k));
}

template <int TYPE>
static int launch_f16_type(rcu_ctx *ctx, const __half *bact, const float *tok_scale, const ActsView &a,
                           const HostJob *jobs, int n_jobs) {
    constexpr uint32_t BOX = raw_box_c<TYPE>();
    HParams p{};
    HMaps maps{};
    uint64_t tiles = 0;
    for (int i = 0; i < n_jobs; i++) {
        const rcu_weight *w = jobs[i].w;
        p.job[i] = HJob{jobs[i].out, jobs[i].ld, (uint32_t)w->rows, (uint32_t)tiles};
        tiles += (w->rows + kHRows - 1) / kHRows;
        if (int st = make_map_2d(ctx, &maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, w->data, w->row_bytes / 2, w->rows,
                                 w->row_bytes, BOX / 2, kHRows, CU_TENSOR_MAP_SWIZZLE_NONE))
            return st;
    }
    if (tiles >= (1u << 31)) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: too many row tiles");
    uint32_t nt = 0, splits = 1;
    pick_tiling(tiles, a.n_tok, a.k / QK_K, n_jobs == 1 ? jobs[0].w->rows : 0, ctx->num_sms, &nt, &splits);
    if (splits > 1) {
        const size_t part = (size_t)splits * a.n_tok * jobs[0].w->rows * sizeof(float);
        const size_t cnt = (size_t)tiles * ((a.n_tok + nt - 1) / nt) * sizeof(uint32_t);
        if (int st = ensure_split_scratch(ctx, part, cnt)) return st;
        p.part = reinterpret_cast<float *>(ctx->k_part);
        p.cnt = ctx->k_cnt;
    }
    p.splits = splits;
    p.n_jobs = (uint32_t)n_jobs;
    p.tok_scale = tok_scale;
    p.k = a.k;
    p.n_tok = a.n_tok;
    p.nt = nt;
    // D f32, A and B f16, both K-major, N = nt, M = 128
    p.idesc = (1u << 4) | ((nt >> 3) << 17) | ((uint32_t)(kHRows >> 4) << 24);
    p.early = ctx->early_weights ? 1 : 0;
    p.err = ctx->dev_err;
    CUtensorMap mb;
    if (int st = make_map_2d(ctx, &mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, bact, a.k, a.n_tok, (uint64_t)a.k * 2, 64, nt,
                             CU_TENSOR_MAP_SWIZZLE_128B))
        return st;
    const size_t smem = sizeof(HSmem) + 1024;
    RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_gemm_f16<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const dim3 grid((uint32_t)tiles, (a.n_tok + nt - 1) / nt, splits);
    RCU_CUDA_TRY(ctx, launch_k(ctx, k_gemm_f16<TYPE>, grid, dim3(kHThreads), smem, maps, mb, p));
    return RCU_OK;
}

static int launch_f16_group(rcu_ctx *ctx, const __half *bact, const float *ts, const ActsView &a, const HostJob *jobs,
                            int n) {
    switch (jobs[0].w->type) {
        case T_Q4_0: return launch_f16_type<T_Q4_0>(ctx, bact, ts, a, jobs, n);
        case T_Q4_1: return launch_f16_type<T_Q4_1>(ctx, bact, ts, a, jobs, n);
        case T_Q5_0: return launch_f16_type<T_Q5_0>(ctx, bact, ts, a, jobs, n);
        case T_Q5_1: return launch_f16_type<T_Q5_1>(ctx, bact, ts, a, jobs, n);
        case T_Q8_0: return launch_f16_type<T_Q8_0>(ctx, bact, ts, a, jobs, n);
        case T_Q4_K: return launch_f16_type<T_Q4_K>(ctx, bact, ts, a, jobs, n);
        case T_Q5_K: return launch_f16_type<T_Q5_K>(ctx, bact, ts, a, jobs, n);
        case T_Q6_K: return launch_f16_type<T_Q6_K>(ctx, bact, ts, a, jobs, n);
        default: return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: type");
    }
}

int launch_gemm_f16(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs) {
    if (sizeof(HSmem) + 1024 > ctx->max_smem_optin) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: smem");
    for (int i = 0; i < n_jobs; i++)
        if (!gemm_f16_ok(a, jobs[i])) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: type or shape not supported");
    if (int st = ensure_f16_scratch(ctx, f16_scratch_bytes(a.n_tok, a.k))) return st;
    __half *bact = reinterpret_cast<__half *>(ctx->h_act);
    float *ts = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ctx->h_act) +
                                          (f16_scratch_bytes(a.n_tok, a.k) - (size_t)a.n_tok * 4));
    uint32_t done_fmt = 0;
    for (int i = 0; i < n_jobs;) {
        const uint32_t fmt = act_format(jobs[i].w->type);
        if (fmt != done_fmt) {  // jobs of one format share the f16 activations
            RCU_CUDA_TRY(ctx, launch_k(ctx, k_acts_f16, dim3(a.n_tok), dim3(kActsF16Threads), 0, a, fmt, bact, ts,
                                       (const uint32_t *)nullptr));
            done_fmt = fmt;
        }
        int n = 1;  // consecutive jobs of the same type share a launch
        while (i + n < n_jobs && n < kF16MaxJobs && jobs[i + n].w->type == jobs[i].w->type) n++;
        if (int st = launch_f16_group(ctx, bact, ts, a, jobs + i, n)) return st;
        i += n;
    }
    return RCU_OK;
}

// ---- grouped launches (mixture of experts) --------------------------------------------------
bool gemm_f16_grouped_ok(const rcu_weight *w, uint32_t k, uint32_t n_exp, uint32_t grp_rows) {
    return gemv_supported(w->type) && k % QK_K == 0 && (w->row_bytes & 15) == 0 && (((uintptr_t)w->data) & 15) == 0 &&
           n_exp >= 1 && n_exp <= kGrpMaxExperts && w->rows == (uint64_t)n_exp * grp_rows && w->cols == k;
}

int gemm_f16_gather(rcu_ctx *ctx, const ActsView &a, uint32_t fmt, const uint32_t *src_rows, uint32_t n_rows,
                    const __half **act, const float **scale) {
    if (int st = ensure_f16_scratch(ctx, f16_scratch_bytes(n_rows, a.k))) return st;
    __half *bact = reinterpret_cast<__half *>(ctx->h_act);
    float *ts = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ctx->h_act) +
                                          (f16_scratch_bytes(n_rows, a.k) - (size_t)n_rows * 4));
    if (n_rows)
        RCU_CUDA_TRY(ctx, launch_k(ctx, k_acts_f16, dim3(n_rows), dim3(kActsF16Threads), 0, a, fmt, bact, ts, src_rows));
    *act = bact;
    *scale = ts;
    return RCU_OK;
}

template <int TYPE>
static int launch_grouped_type(rcu_ctx *ctx, const __half *act, const float *scale, uint32_t n_rows, uint32_t k,
                               const HostJob *jobs, int n_jobs, uint32_t grp_rows, const uint32_t *off, uint32_t n_exp) {
    constexpr uint32_t BOX = raw_box_c<TYPE>();
    const uint32_t rtiles = (grp_rows + kHRows - 1) / kHRows;
    // tokens per CTA: the fewest waves over the (expert, token tile) items
    uint32_t nt = 0, n_items = 0;
    double best = 1e300;
    for (uint32_t cand : {64u, 128u, 256u}) {
        uint64_t items = 0;
        for (uint32_t e = 0; e < n_exp; e++) items += (off[e + 1] - off[e] + cand - 1) / cand;
        if (items > (uint64_t)kGrpMaxItems) continue;
        const uint64_t ctas = items * rtiles * (uint64_t)n_jobs;
        const double cost = (double)((ctas + ctx->num_sms - 1) / ctx->num_sms) * (cand + 64);
        if (cost < best) best = cost, nt = cand, n_items = (uint32_t)items;
    }
    if (!nt) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: too many expert token tiles");
    if (n_items == 0) return RCU_OK;
    HParams p{};
    HMaps maps{};
    for (int i = 0; i < n_jobs; i++) {
        const rcu_weight *w = jobs[i].w;
        p.job[i] = HJob{jobs[i].out, jobs[i].ld, grp_rows, (uint32_t)(i * rtiles)};
        if (int st = make_map_2d(ctx, &maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, w->data, w->row_bytes / 2, w->rows,
                                 w->row_bytes, BOX / 2, kHRows, CU_TENSOR_MAP_SWIZZLE_NONE))
            return st;
    }
    uint32_t it = 0;
    for (uint32_t e = 0; e < n_exp; e++)
        for (uint32_t t0 = 0; t0 < off[e + 1] - off[e]; t0 += nt, it++) {
            p.grp_exp[it] = (uint16_t)e;
            p.grp_tile[it] = (uint16_t)(t0 / nt);
        }
    for (uint32_t e = 0; e <= n_exp; e++) p.grp_off[e] = off[e];
    p.grp = n_items;
    p.grp_rows = grp_rows;
    p.splits = 1;
    p.tok_scale = scale;
    p.n_jobs = (uint32_t)n_jobs;
    p.k = k;
    p.n_tok = n_rows;
    p.nt = nt;
    p.idesc = (1u << 4) | ((nt >> 3) << 17) | ((uint32_t)(kHRows >> 4) << 24);
    p.early = 0;  // the expert choice was made on this pass
    p.err = ctx->dev_err;
    CUtensorMap mb;
    if (int st = make_map_2d(ctx, &mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, k, n_rows, (uint64_t)k * 2, 64, nt,
                             CU_TENSOR_MAP_SWIZZLE_128B))
        return st;
    const size_t smem = sizeof(HSmem) + 1024;
    RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_gemm_f16<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const dim3 grid(rtiles * (uint32_t)n_jobs, n_items);
    RCU_CUDA_TRY(ctx, launch_k(ctx, k_gemm_f16<TYPE>, grid, dim3(kHThreads), smem, maps, mb, p));
    return RCU_OK;
}

int launch_gemm_f16_grouped(rcu_ctx *ctx, const __half *act, const float *scale, uint32_t n_rows, uint32_t k,
                            const HostJob *jobs, int n_jobs, uint32_t grp_rows, const uint32_t *off, uint32_t n_exp) {
    if (n_jobs < 1 || n_jobs > kF16MaxJobs) return set_err(ctx, RCU_ERR_INVALID, "gemm: 1..4 grouped jobs");
    for (int i = 0; i < n_jobs; i++)
        if (jobs[i].w->type != jobs[0].w->type || !gemm_f16_grouped_ok(jobs[i].w, k, n_exp, grp_rows))
            return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: grouped expert shape not supported");
    switch (jobs[0].w->type) {
        case T_Q4_0: return launch_grouped_type<T_Q4_0>(ctx, act, scale, n_rows, k, jobs, n_jobs, grp_rows, off, n_exp);
        case T_Q4_1: return launch_grouped_type<T_Q4_1>(ctx, act, scale, n_rows, k, jobs, n_jobs, grp_rows, off, n_exp);
        case T_Q5_0: return launch_grouped_type<T_Q5_0>(ctx, act, scale, n_rows, k, jobs, n_jobs, grp_rows, off, n_exp);
        case T_Q5_1: return launch_grouped_type<T_Q5_1>(ctx, act, scale, n_rows, k, jobs, n_jobs, grp_rows, off, n_exp);
        case T_Q8_0: return launch_grouped_type<T_Q8_0>(ctx, act, scale, n_rows, k, jobs, n_jobs, grp_rows, off, n_exp);
        case T_Q4_K: return launch_grouped_type<T_Q4_K>(ctx, act, scale, n_rows, k, jobs, n_jobs, grp_rows, off, n_exp);
        case T_Q5_K: return launch_grouped_type<T_Q5_K>(ctx, act, scale, n_rows, k, jobs, n_jobs, grp_rows, off, n_exp);
        case T_Q6_K: return launch_grouped_type<T_Q6_K>(ctx, act, scale, n_rows, k, jobs, n_jobs, grp_rows, off, n_exp);
        default: return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: type");
    }
}

}  // namespace rcu
