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
//               per operand stage into one f32 accumulator of NT columns;
//   * warps 2-9 dequantize: two threads per weight row, 32 values each per operand stage,
//               written as f16 into the canonical 128B-swizzled K-major layout; after the last
//               stage the same warps read the accumulator (tcgen05.ld) and store Y.
// Up to kF16MaxJobs weights sharing the activations (q/k/v, gate/up) run in one launch: the
// grid's x dimension walks the row tiles of each job in turn.
// All waits are bounded; TMEM is freed on every exit path.
#include <cuda.h>

#include <algorithm>

#include "rcu_blocks.cuh"
#include "rcu_kernels.h"
#include "rcu_tc.cuh"

namespace rcu {

constexpr int kHRows = 128;        // weight rows per CTA (MMA M)
constexpr int kHMaxTok = 256;      // tokens per CTA at most (MMA N)
constexpr int kHStages = 3;        // operand stages (K 64 each)
constexpr int kHRawStages = 2;     // raw GGUF stages (K 256 each)
constexpr int kHRawMax = 272;      // raw bytes per row per stage at most (Q8_0: 8 x 34)
constexpr int kHUnpackWarps = 8;
constexpr int kHThreads = (2 + kHUnpackWarps) * 32;
constexpr int kF16MaxJobs = 4;
constexpr uint32_t kF16MinTok = 32;  // below this the 8-token GEMV slices are used

struct HSmem {
    uint8_t a[kHStages][kHRows * 128];      // f16 weights, 8 rows x 128 B swizzle atoms
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
    uint32_t n_jobs, k, n_tok, nt, idesc;
    int early;  // weights may be loaded before the grid dependency wait
    uint32_t *err;
};

// ---- dequantization of 32 values of one row -----------------------------------------------
template <int TYPE>
constexpr uint32_t unit_bytes_c() {  // bytes of 256 values of K
    return TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : TYPE == T_Q6_K ? 210 : 8 * blk_bytes_c<TYPE>();
}
// Raw stage box per row: Q6_K superblocks (210 B) start on even, not 16-byte, offsets, so its
// box starts at the 16-byte boundary below and is wide enough for any start within 16 bytes.
template <int TYPE>
constexpr uint32_t raw_box_c() {
    return TYPE == T_Q6_K ? 240 : unit_bytes_c<TYPE>();
}

// Byte b of w as the exact float (byte - bias): the byte is placed in the mantissa of 2^23.
__device__ __forceinline__ float bytef(uint32_t w, uint32_t b, float c0) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | b)) - c0;
}
__device__ __forceinline__ uint32_t h2u(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Values [32 j, 32 j + 32) of the 256-value unit that starts `ofs` bytes into `row` (a 16-byte
// aligned row of a raw stage), dequantized as reference.rs:53-207 defines them.
template <int TYPE>
__device__ __forceinline__ void dq32(const uint8_t *row, uint32_t ofs, uint32_t j, float (&v)[32]) {
    if constexpr (TYPE == T_Q4_0 || TYPE == T_Q4_1 || TYPE == T_Q5_0 || TYPE == T_Q5_1 || TYPE == T_Q8_0) {
        BlkW b;
        dec_blk<TYPE>(row, j * blk_bytes_c<TYPE>(), b);
        constexpr float bias = TYPE == T_Q4_0 ? 8.0f : TYPE == T_Q5_0 ? 16.0f : TYPE == T_Q8_0 ? 128.0f : 0.0f;
        constexpr float c0 = 8388608.0f + bias;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t w = b.v[i];
            if ((TYPE == T_Q4_0 || TYPE == T_Q4_1) && i >= 4) w >>= 4;  // 16 x high nibble -> nibble
            if (TYPE == T_Q8_0) w ^= 0x80808080u;                        // int8 -> q + 128
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float q = bytef(w, e, c0);
                v[4 * i + e] = (TYPE == T_Q4_1 || TYPE == T_Q5_1) ? fmaf(q, b.d, b.m) : q * b.d;
            }
        }
    } else if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        // d, dmin, 12 scale bytes, [Q5_K: qh 32 B], qs 128 B (reference.rs:153-189)
        const uint32_t *w = reinterpret_cast<const uint32_t *>(row);
        const uint32_t h0 = w[0];
        // get_scale_min_k4 (reference.rs:8-14) with a runtime j and no indexed array
        const uint32_t sh = 8 * (j & 3);
        const uint32_t b0 = (w[1] >> sh) & 0xffu, b1 = (w[2] >> sh) & 0xffu, b2 = (w[3] >> sh) & 0xffu;
        const uint32_t sc = j < 4 ? b0 & 63u : (b2 & 0xFu) | ((b0 >> 6) << 4);
        const uint32_t mn = j < 4 ? b1 & 63u : (b2 >> 4) | ((b1 >> 6) << 4);
        const float ds = f16_bits_to_f32(h0) * (float)sc, dm = f16_bits_to_f32(h0 >> 16) * (float)mn;
        constexpr uint32_t qs_word = TYPE == T_Q4_K ? 4 : 12;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t qw = w[qs_word + 8 * (j >> 1) + i];
            uint32_t q = (j & 1) ? (qw >> 4) & 0x0F0F0F0Fu : qw & 0x0F0F0F0Fu;
            if (TYPE == T_Q5_K) q |= ((w[4 + i] >> j) & 0x01010101u) << 4;  // bit j of qh[l]
#pragma unroll
            for (int e = 0; e < 4; e++) v[4 * i + e] = fmaf(bytef(q, e, 8388608.0f), ds, -dm);
        }
    } else {  // Q6_K: ql 128 B, qh 64 B, 16 int8 scales, d (reference.rs:190-207)
        const uint32_t n = j >> 2, jj = j & 3;
        uint32_t ql[8], qh[8];
        ld_words<8>(row, ofs + 64 * n + 32 * (jj & 1), ql);
        ld_words<8>(row, ofs + 128 + 32 * n, qh);
        const float d = __half2float(*reinterpret_cast<const __half *>(row + ofs + 208));
        const float ds0 = d * (float)(int8_t)row[ofs + 192 + 8 * n + 2 * jj];
        const float ds1 = d * (float)(int8_t)row[ofs + 193 + 8 * n + 2 * jj];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t lo = jj < 2 ? ql[i] & 0x0F0F0F0Fu : (ql[i] >> 4) & 0x0F0F0F0Fu;
            const uint32_t q = lo | (((qh[i] >> (2 * jj)) & 0x03030303u) << 4);
#pragma unroll
            for (int e = 0; e < 4; e++) v[4 * i + e] = bytef(q, e, 8388608.0f + 32.0f) * (i < 4 ? ds0 : ds1);
        }
    }
}

// 32 f16 values of row r as 16-byte chunks c0..c0+3 of a 128B-swizzled K-major tile.
__device__ __forceinline__ void store_chunks(uint8_t *tile, uint32_t r, uint32_t c0, const float (&v)[32]) {
    uint8_t *rowp = tile + r * 128;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint4 q = make_uint4(h2u(v[8 * i], v[8 * i + 1]), h2u(v[8 * i + 2], v[8 * i + 3]),
                                   h2u(v[8 * i + 4], v[8 * i + 5]), h2u(v[8 * i + 6], v[8 * i + 7]));
        *reinterpret_cast<uint4 *>(rowp + (((c0 + i) ^ (r & 7)) << 4)) = q;
    }
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)acc)
        : "memory");
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
    const uint32_t n0 = (blockIdx.x - jb.tile0) * kHRows, m0 = blockIdx.y * p.nt;
    const uint32_t n_unit = p.k / QK_K, n_it = n_unit * 4;

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
    if (warp == 1) tmem_alloc<kHMaxTok>(&S.tmem_base);
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
                tma_load_2d(S.raw[rs], mw, (int)(((u * UB) & ~15u) >> 1), (int)n0, &S.raw_full[rs]);
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
                tma_load_2d(S.b[s], &map_b, (int)(it * 64), (int)m0, &S.b_full[s]);
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
                    mma_f16(tmem, sw128_desc(S.a[s] + 32 * kk), sw128_desc(S.b[s] + 32 * kk), p.idesc, (it | kk) != 0);
                mma_commit(&S.ab_empty[s]);
            }
            mma_commit(&S.acc_full);  // also on an early exit: tracks every MMA issued
        }
    } else {  // ---- dequantize, then epilogue (warps 2-9) ----
        const uint32_t ut = threadIdx.x - 64, r = ut & (kHRows - 1), h = ut / kHRows;
        bool ok = true;
        for (uint32_t it = 0; it < n_it; it++) {
            const uint32_t u = it >> 2, g = it & 3, rs = u % kHRawStages, s = it % kHStages;
            if (g == 0 && !warp_wait(&S.raw_full[rs], (u / kHRawStages) & 1, p.err, ERR_TIMEOUT_FULL)) {
                ok = false;
                break;
            }
            if (it >= kHStages && !warp_wait(&S.ab_empty[s], ((it / kHStages) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
                ok = false;
                break;
            }
            float v[32];
            dq32<TYPE>(S.raw[rs] + r * BOX, (u * UB) & 15u, 2 * g + h, v);
            store_chunks(S.a[s], r, 4 * h, v);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&S.a_full[s]);
                if (g == 3) mbar_arrive(&S.raw_empty[rs]);
            }
        }
        pdl_wait();  // the output may still be read by the kernel before this one
        if (ok && warp_wait(&S.acc_full, 0, p.err, ERR_TIMEOUT_FULL)) {
            tc_fence_after();
            const uint32_t q = warp & 3, hh = (warp - 2) >> 2, half = p.nt / 2;
            const uint32_t n = n0 + 32 * q + lane;
            for (uint32_t c = hh * half; c < (hh + 1) * half; c += 32) {
                uint32_t x[32];
                tmem_ld32(tmem + ((32 * q) << 16) + c, x);
                tmem_wait_ld();
                if (n < jb.rows) {
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        const uint32_t m = m0 + c + e;
                        if (m < p.n_tok) jb.out[(uint64_t)m * jb.ld + n] = __uint_as_float(x[e]);
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
        tmem_free<kHMaxTok>(tmem);
    }
}

// A[t][k] = f16(d_a * q_a) of the prepared Q8_0 or Q8_K activations (8 values per thread).
__global__ void k_acts_f16(const ActsView a, uint32_t fmt, __half *__restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const uint64_t n8 = (uint64_t)a.n_tok * a.k / 8;
    const int8_t *qs = fmt == RCU_ACT_Q8_0 ? a.q0 : a.qk;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t e0 = i * 8, t = e0 / a.k;
        const uint32_t kk = (uint32_t)(e0 - t * a.k);
        const uint2 c = *reinterpret_cast<const uint2 *>(qs + e0);
        const float d = fmt == RCU_ACT_Q8_0 ? a.d0[t * (a.k / QK) + kk / QK] : a.dk[t * (a.k / QK_K) + kk / QK_K];
        uint4 o;
        o.x = h2u((float)sbyte(c.x, 0) * d, (float)sbyte(c.x, 1) * d);
        o.y = h2u((float)sbyte(c.x, 2) * d, (float)sbyte(c.x, 3) * d);
        o.z = h2u((float)sbyte(c.y, 0) * d, (float)sbyte(c.y, 1) * d);
        o.w = h2u((float)sbyte(c.y, 2) * d, (float)sbyte(c.y, 3) * d);
        *reinterpret_cast<uint4 *>(out + e0) = o;
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

// Tokens per CTA: the fewest waves of CTAs, a tile of nt tokens costing about nt + 64 (the
// dequantization of the weight tile is paid once per token tile).
static uint32_t pick_nt(uint64_t tiles_w, uint32_t n_tok, int sms) {
    uint32_t best = 64;
    double best_cost = 1e300;
    for (uint32_t nt : {256u, 192u, 128u, 64u}) {
        const uint64_t ctas = tiles_w * ((n_tok + nt - 1) / nt);
        const double cost = (double)((ctas + sms - 1) / sms) * (nt + 64);
        if (cost < best_cost) {
            best_cost = cost;
            best = nt;
        }
    }
    return best;
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

int gemm_f16_reserve(rcu_ctx *ctx, uint64_t n_tok, uint64_t k) { return ensure_f16_scratch(ctx, n_tok * k * 2); }

template <int TYPE>
static int launch_f16_type(rcu_ctx *ctx, const __half *bact, const ActsView &a, const HostJob *jobs, int n_jobs) {
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
    const uint32_t nt = pick_nt(tiles, a.n_tok, ctx->num_sms);
    p.n_jobs = (uint32_t)n_jobs;
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
    const dim3 grid((uint32_t)tiles, (a.n_tok + nt - 1) / nt);
    RCU_CUDA_TRY(ctx, launch_k(ctx, k_gemm_f16<TYPE>, grid, dim3(kHThreads), smem, maps, mb, p));
    return RCU_OK;
}

static int launch_f16_group(rcu_ctx *ctx, const __half *bact, const ActsView &a, const HostJob *jobs, int n) {
    switch (jobs[0].w->type) {
        case T_Q4_0: return launch_f16_type<T_Q4_0>(ctx, bact, a, jobs, n);
        case T_Q4_1: return launch_f16_type<T_Q4_1>(ctx, bact, a, jobs, n);
        case T_Q5_0: return launch_f16_type<T_Q5_0>(ctx, bact, a, jobs, n);
        case T_Q5_1: return launch_f16_type<T_Q5_1>(ctx, bact, a, jobs, n);
        case T_Q8_0: return launch_f16_type<T_Q8_0>(ctx, bact, a, jobs, n);
        case T_Q4_K: return launch_f16_type<T_Q4_K>(ctx, bact, a, jobs, n);
        case T_Q5_K: return launch_f16_type<T_Q5_K>(ctx, bact, a, jobs, n);
        case T_Q6_K: return launch_f16_type<T_Q6_K>(ctx, bact, a, jobs, n);
        default: return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: type");
    }
}

int launch_gemm_f16(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs) {
    if (sizeof(HSmem) + 1024 > ctx->max_smem_optin) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: smem");
    for (int i = 0; i < n_jobs; i++)
        if (!gemm_f16_ok(a, jobs[i])) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: type or shape not supported");
    if (int st = ensure_f16_scratch(ctx, (size_t)a.n_tok * a.k * 2)) return st;
    __half *bact = reinterpret_cast<__half *>(ctx->h_act);
    const uint64_t n8 = (uint64_t)a.n_tok * a.k / 8;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n8 + 255) / 256, (uint64_t)ctx->num_sms * 8);
    uint32_t done_fmt = 0;
    for (int i = 0; i < n_jobs;) {
        const uint32_t fmt = act_format(jobs[i].w->type);
        if (fmt != done_fmt) {  // jobs of one format share the f16 activations
            RCU_CUDA_TRY(ctx, launch_k(ctx, k_acts_f16, dim3(blocks), dim3(256), 0, a, fmt, bact));
            done_fmt = fmt;
        }
        int n = 1;  // consecutive jobs of the same type share a launch
        while (i + n < n_jobs && n < kF16MaxJobs && jobs[i + n].w->type == jobs[i].w->type) n++;
        if (int st = launch_f16_group(ctx, bact, a, jobs + i, n)) return st;
        i += n;
    }
    return RCU_OK;
}

}  // namespace rcu
