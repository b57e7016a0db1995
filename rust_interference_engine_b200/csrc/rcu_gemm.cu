// rcu_gemm.cu -- prefill GEMM (n_tok >= 32) with the reference's exact int8 block sums, on the
// 5th-generation tensor cores (Q4_0 weights x Q8_0 activations).
//
// Y[t][n] = sum_b d_a[t][b] * d_w[n][b] * S_b[t][n], with S_b the exact int32 dot of block b
// (the reference forms the same per-block ints one row at a time:
// crates/rie-core/src/kernels/matmul.rs:178-241 via vec_dot / vec_dot_x4,
// crates/rie-core/src/quant/reference.rs:221-293).
//
// Roofline: one tcgen05 kind::i8 MMA (M 128, N 128, K 32) per block forms every S_b of a tile,
// but each S_b then needs its own f32 scaling -- two FMAs per output per 32 values of K -- so
// the FP32 work (128 FMA per clock per SM) bounds the kernel, not the tensor pipe. Measured, the
// round trip of each block (MMA commit -> epilogue -> re-arm) is the larger cost.
//
// Per CTA: a 128-weight-row x 128-token output tile; the grid walks the row tiles of up to
// four weights that share the activations (q/k/v, gate/up) in one launch.
//   * warp 0    TMA producer: raw GGUF rows (8 blocks = K 256 per stage), int8 activation codes
//               (128B-swizzled, K-major) and the activation block scales; 2 operand stages,
//               released by the MMA commit;
//   * warps 1-2 unpack: GGUF blocks -> int8 weight tile in the 128B-swizzled K-major layout
//               the tensor core reads; the block scales d_w and the transposed d_a go to a
//               4-slot scale ring that only the epilogue releases;
//   * warp 3    MMA issuer: one tcgen05.mma.kind::i8 per block, two blocks per commit, into
//               one of two TMEM accumulator pairs (2 x 128 columns each, the whole tensor
//               memory), so the tensor core runs up to four blocks ahead of the epilogue;
//   * warps 4-19 epilogue: warp w reads TMEM lanes 32*(w%4).. and one quarter of the tokens,
//               for both blocks of a pair: tcgen05.ld of the block's 32 int32 sums, the FMAs
//               below, then re-arm the accumulator with the f32
//               magic 1.5*2^23 (the next block's int sum S then reads back as the float
//               1.5*2^23 + S exactly), and two packed FMAs per pair of outputs:
//               t = fma(X, d_w, -1.5*2^23*d_w) = round(S * d_w), acc = fma(t, d_a, acc).
// All waits are bounded; TMEM is freed on every exit path.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cstring>

#include "rcu_kernels.h"
#include "rcu_tc.cuh"

namespace rcu {

constexpr int kTileN = 128;        // weight rows per CTA (MMA M, TMEM lanes)
constexpr int kTileM = 128;        // tokens per CTA (MMA N)
constexpr int kStageBlocks = 8;    // 32-value blocks per operand stage (K = 256)
constexpr int kStages = 2;         // operand stages (raw weights, unpacked weights, activations)
constexpr int kScaleSlots = 4;     // scale ring (d_w, transposed d_a), one slot per stage
constexpr int kTBufs = 2;          // TMEM accumulator pairs: two blocks of 128 columns each
constexpr int kEpiWarps = 16;
constexpr int kEpiWarp0 = 4;       // warps: 0 producer, 1-2 unpack, 3 MMA, 4.. epilogue
constexpr int kGemmThreads = (kEpiWarp0 + kEpiWarps) * 32;
constexpr int kRawBox = kStageBlocks * 18;  // Q4_0 bytes per row per stage (144, 16-byte multiple)
constexpr int kMaxI8Jobs = 4;
constexpr uint32_t kGemmMinTok = 32;  // below this the 8-token GEMV slices are faster
constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;

struct GemmSmem {
    // 1024-aligned operand tiles first
    uint8_t a[kStages][2][kTileN * 128];   // unpacked weights, 2 swizzle atoms of K 128
    uint8_t b[kStages][2][kTileM * 128];   // activation codes (TMA, 128B swizzle)
    uint8_t raw[kStages][kTileN * kRawBox];
    float da[kStages][kTileM][kStageBlocks];      // activation block scales as TMA lands them
    float daT[kScaleSlots][kStageBlocks][kTileM];  // ... transposed: one block's 128 tokens contiguous
    float dw[kScaleSlots][kStageBlocks][kTileN];
    uint64_t full[kStages], unpacked[kStages], empty[kStages];
    uint64_t sfull[kScaleSlots], sempty[kScaleSlots];
    uint64_t tfull[kTBufs], tempty[kTBufs];  // one handoff per pair of blocks
    uint32_t tmem_base;
};

struct I8Job {
    float *out;
    uint64_t ld;
    uint32_t rows, tile0;  // weight rows; first grid-x tile of this job
};
struct I8Maps {
    CUtensorMap w[kMaxI8Jobs];  // raw GGUF bytes [rows][row_bytes] of each job
};
struct GemmParams {
    I8Job job[kMaxI8Jobs];
    uint32_t n_jobs, k, n_tok;
    uint32_t *err;
};

// Instruction descriptor: D s32, A s8, B s8, both K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTileM >> 3) << 17) |
                            ((uint32_t)(kTileN >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, 1, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(kIdesc)
        : "memory");
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(r)
        : "l"(*reinterpret_cast<uint64_t *>(&a)), "l"(*reinterpret_cast<uint64_t *>(&b)),
          "l"(*reinterpret_cast<uint64_t *>(&c)));
    return *reinterpret_cast<float2 *>(&r);
}

// A raw row of 8 Q4_0 blocks (144 bytes) as 36 words: 9 16-byte loads, conflict-free for the
// 8 lanes of a load phase (row stride 144 B = 9 chunks, odd).
__device__ __forceinline__ void load_raw_row(const uint8_t *row, uint32_t (&w)[36]) {
#pragma unroll
    for (int i = 0; i < 9; i++) {
        const uint4 v = *reinterpret_cast<const uint4 *>(row + 16 * i);
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
    }
}
// Block J of the row (bytes 18J..18J+17): its f32 scale and 32 int8 codes (nib - 8) in element
// order as two 16-byte chunks. J is a compile-time constant, so every shift is one too.
template <int J>
__device__ __forceinline__ void unpack_q4_0(const uint32_t (&w)[36], uint4 &c0, uint4 &c1, float &d) {
    constexpr int W = (18 * J) / 4;  // word holding the scale
    uint32_t q[4];
    if ((J & 1) == 0) {  // scale in the low half of word W, nibbles from byte 2 of it
        d = f16_bits_to_f32(w[W] & 0xFFFFu);
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = __funnelshift_r(w[W + i], w[W + i + 1], 16);
    } else {  // scale in the high half of word W, nibbles word-aligned after it
        d = f16_bits_to_f32(w[W] >> 16);
#pragma unroll
        for (int i = 0; i < 4; i++) q[i] = w[W + 1 + i];
    }
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        // nibble -> int8 (nib - 8): flip bit 3 then sign-extend the 4-bit value
        const uint32_t l = (q[i] & 0x0F0F0F0Fu) ^ 0x08080808u, h = ((q[i] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        lo[i] = l | ((l & 0x08080808u) * 30u);
        hi[i] = h | ((h & 0x08080808u) * 30u);
    }
    c0 = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    c1 = make_uint4(hi[0], hi[1], hi[2], hi[3]);
}
template <int J>
__device__ __forceinline__ void unpack_store(const uint32_t (&w)[36], uint8_t *a0, uint8_t *a1, uint32_t r,
                                             float *dw_j0) {
    uint4 c0, c1;
    float d;
    unpack_q4_0<J>(w, c0, c1, d);
    uint8_t *rowp = (J < 4 ? a0 : a1) + r * 128;
    constexpr uint32_t ch = 2 * (J & 3);
    *reinterpret_cast<uint4 *>(rowp + (((ch) ^ (r & 7)) << 4)) = c0;
    *reinterpret_cast<uint4 *>(rowp + (((ch + 1) ^ (r & 7)) << 4)) = c1;
    dw_j0[J * kTileN + r] = d;
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_i8(const __grid_constant__ I8Maps maps, const __grid_constant__ CUtensorMap map_a,
              const __grid_constant__ CUtensorMap map_da, const __grid_constant__ GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    GemmSmem &S = *reinterpret_cast<GemmSmem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t ji = 0;
    while (ji + 1 < p.n_jobs && blockIdx.x >= p.job[ji + 1].tile0) ji++;
    const I8Job &jb = p.job[ji];
    const uint32_t n0 = (blockIdx.x - jb.tile0) * kTileN, m0 = blockIdx.y * kTileM;
    const uint32_t n_iter = p.k / QK / kStageBlocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.unpacked[s], 2);
            mbar_init(&S.empty[s], 1);  // the MMA commit of the stage's blocks
        }
        for (int j = 0; j < kScaleSlots; j++) {
            mbar_init(&S.sfull[j], 2);
            mbar_init(&S.sempty[j], kEpiWarps);
        }
        for (int b = 0; b < kTBufs; b++) {
            mbar_init(&S.tfull[b], 1);
            mbar_init(&S.tempty[b], kEpiWarps);
        }
        fence_mbar_init();
    }
    if (warp == 3) tmem_alloc<kTBufs * 256>(&S.tmem_base);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    const int q = warp & 3, cq = (warp - kEpiWarp0) >> 2;  // epilogue: TMEM lane quarter, token quarter

    if (warp >= kEpiWarp0) {  // arm every accumulator with the magic offset
        for (int b = 0; b < 2 * kTBufs; b++) tmem_st32_const(tmem + ((uint32_t)(32 * q) << 16) + b * 128 + 32 * cq, kMagicBits);
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 0) {  // ---- TMA producer ----
        if (lane == 0) {
            const CUtensorMap *mw = &maps.w[ji];
            for (uint32_t it = 0; it < n_iter; it++) {
                const uint32_t s = it % kStages;
                if (it >= kStages && !mbar_wait_sleep(&S.empty[s], ((it / kStages) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY))
                    break;
                constexpr uint32_t bytes = kTileN * kRawBox + 2 * kTileM * 128 + kTileM * kStageBlocks * 4;
                mbar_arrive_expect_tx(&S.full[s], bytes);
                tma_load_2d(S.raw[s], mw, (int)(it * kRawBox), (int)n0, &S.full[s]);
                tma_load_2d(S.b[s][0], &map_a, (int)(it * 256), (int)m0, &S.full[s]);
                tma_load_2d(S.b[s][1], &map_a, (int)(it * 256 + 128), (int)m0, &S.full[s]);
                tma_load_2d(S.da[s], &map_da, (int)(it * kStageBlocks), (int)m0, &S.full[s]);
            }
        }
    } else if (warp <= 2) {  // ---- unpack (64 threads: weight rows r and r + 64, their tokens' scales) ----
        const uint32_t t = threadIdx.x - 32;
        for (uint32_t it = 0; it < n_iter; it++) {
            const uint32_t s = it % kStages, slot = it % kScaleSlots;
            if (!mbar_wait_sleep(&S.full[s], (it / kStages) & 1, p.err, ERR_TIMEOUT_FULL)) break;
            if (it >= kScaleSlots &&
                !mbar_wait_sleep(&S.sempty[slot], ((it / kScaleSlots) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY))
                break;
#pragma unroll 1
            for (uint32_t r = t; r < kTileN; r += 64) {
                uint32_t w[36];
                load_raw_row(S.raw[s] + r * kRawBox, w);
                uint8_t *a0 = S.a[s][0], *a1 = S.a[s][1];
                float *dwp = &S.dw[slot][0][0];
                unpack_store<0>(w, a0, a1, r, dwp);
                unpack_store<1>(w, a0, a1, r, dwp);
                unpack_store<2>(w, a0, a1, r, dwp);
                unpack_store<3>(w, a0, a1, r, dwp);
                unpack_store<4>(w, a0, a1, r, dwp);
                unpack_store<5>(w, a0, a1, r, dwp);
                unpack_store<6>(w, a0, a1, r, dwp);
                unpack_store<7>(w, a0, a1, r, dwp);
                const float4 v0 = *reinterpret_cast<const float4 *>(&S.da[s][r][0]);
                const float4 v1 = *reinterpret_cast<const float4 *>(&S.da[s][r][4]);
                S.daT[slot][0][r] = v0.x;
                S.daT[slot][1][r] = v0.y;
                S.daT[slot][2][r] = v0.z;
                S.daT[slot][3][r] = v0.w;
                S.daT[slot][4][r] = v1.x;
                S.daT[slot][5][r] = v1.y;
                S.daT[slot][6][r] = v1.z;
                S.daT[slot][7][r] = v1.w;
            }
            fence_async_smem();  // the unpacked tile is read by the tensor core (async proxy)
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&S.unpacked[s]);
                mbar_arrive(&S.sfull[slot]);
            }
        }
    } else if (warp == 3) {  // ---- MMA issuer ----
        if (lane == 0) {
            uint32_t b = 0;
            bool ok = true;
            for (uint32_t it = 0; it < n_iter && ok; it++) {
                const uint32_t s = it % kStages;
                if (!mbar_wait_sleep(&S.unpacked[s], (it / kStages) & 1, p.err, ERR_TIMEOUT_FULL) ||
                    !mbar_wait_sleep(&S.full[s], (it / kStages) & 1, p.err, ERR_TIMEOUT_FULL))
                    break;
                tc_fence_after();
                for (int j = 0; j < kStageBlocks; j += 2, b++) {  // b counts pairs of blocks
                    const uint32_t buf = b % kTBufs;
                    if (b >= kTBufs && !mbar_wait_sleep(&S.tempty[buf], ((b / kTBufs) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const uint64_t ad = sw128_desc(S.a[s][(j + h) >> 2] + 32 * ((j + h) & 3));
                        const uint64_t bd = sw128_desc(S.b[s][(j + h) >> 2] + 32 * ((j + h) & 3));
                        mma_i8(tmem + buf * 256 + h * 128, ad, bd);
                    }
                    mma_commit(&S.tfull[buf]);
                }
                mma_commit(&S.empty[s]);
            }
        }
    } else {  // ---- epilogue (warps 4..19) ----
        const uint32_t nrow = 32 * q + lane;  // weight row within the tile
        float2 acc[16];
#pragma unroll
        for (int c = 0; c < 16; c++) acc[c] = make_float2(0.0f, 0.0f);
        uint32_t b = 0;
        bool ok = true;
        for (uint32_t it = 0; it < n_iter && ok; it++) {
            const uint32_t slot = it % kScaleSlots;
            if (!mbar_wait_sleep(&S.sfull[slot], (it / kScaleSlots) & 1, p.err, ERR_TIMEOUT_FULL)) break;
            for (int j = 0; j < kStageBlocks; j += 2, b++) {  // b counts pairs of blocks
                const uint32_t buf = b % kTBufs;
                if (!mbar_wait_sleep(&S.tfull[buf], (b / kTBufs) & 1, p.err, ERR_TIMEOUT_FULL)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int h = 0; h < 2; h++) {
                    const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + buf * 256 + h * 128 + 32 * cq;
                    const float dw = S.dw[slot][j + h][nrow];
                    const float2 dw2 = make_float2(dw, dw), nm2 = make_float2(-kMagic * dw, -kMagic * dw);
                    const float4 *dap = reinterpret_cast<const float4 *>(&S.daT[slot][j + h][32 * cq]);
                    uint32_t x[32];
                    tmem_ld32(ta, x);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float4 d4 = dap[i];
                        const float2 x0 = make_float2(__uint_as_float(x[4 * i]), __uint_as_float(x[4 * i + 1]));
                        const float2 x1 = make_float2(__uint_as_float(x[4 * i + 2]), __uint_as_float(x[4 * i + 3]));
                        acc[2 * i] = ffma2(ffma2(x0, dw2, nm2), make_float2(d4.x, d4.y), acc[2 * i]);
                        acc[2 * i + 1] = ffma2(ffma2(x1, dw2, nm2), make_float2(d4.z, d4.w), acc[2 * i + 1]);
                    }
                    tmem_st32_const(ta, kMagicBits);  // re-arm for the pair after next
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.tempty[buf]);
            }
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(&S.sempty[slot]);
        }
        const uint32_t n = n0 + nrow;
        if (n < jb.rows) {
#pragma unroll
            for (int c = 0; c < 16; c++) {
                const uint32_t m = m0 + 32 * cq + 2 * c;
                if (m < p.n_tok) jb.out[(uint64_t)m * jb.ld + n] = acc[c].x;
                if (m + 1 < p.n_tok) jb.out[(uint64_t)(m + 1) * jb.ld + n] = acc[c].y;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 3) {
        tc_fence_after();
        tmem_free<kTBufs * 256>(tmem);
    }
}

// ---- host side -----------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

int make_map_2d(rcu_ctx *ctx, CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner,
                uint64_t outer, uint64_t stride_bytes, uint32_t box_in, uint32_t box_out, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_err(ctx, RCU_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {stride_bytes};
    const cuuint32_t box[2] = {box_in, box_out};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_err(ctx, RCU_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return RCU_OK;
}

static bool gemm_ok(const ActsView &a, const HostJob &j) {
    const rcu_weight *w = j.w;
    if (w->type != T_Q4_0) return false;  // other types run the f16 GEMM
    if (a.k % 256 != 0 || (w->row_bytes & 15) != 0 || (((uintptr_t)w->data) & 15) != 0) return false;
    return a.n_tok >= kGemmMinTok;
}

// One launch for up to four Q4_0 weights over the same activations.
static int launch_i8_group(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs) {
    GemmParams p{};
    I8Maps maps;
    memset(&maps, 0, sizeof(maps));
    uint32_t tiles = 0;
    for (int i = 0; i < n_jobs; i++) {
        const rcu_weight *w = jobs[i].w;
        p.job[i] = I8Job{jobs[i].out, jobs[i].ld, (uint32_t)w->rows, tiles};
        tiles += (uint32_t)((w->rows + kTileN - 1) / kTileN);
        if (int st = make_map_2d(ctx, &maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, w->data, w->row_bytes, w->rows,
                                 w->row_bytes, kRawBox, kTileN, CU_TENSOR_MAP_SWIZZLE_NONE))
            return st;
    }
    p.n_jobs = (uint32_t)n_jobs;
    p.k = a.k;
    p.n_tok = a.n_tok;
    p.err = ctx->dev_err;
    CUtensorMap ma, mda;
    int st = make_map_2d(ctx, &ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.q0, a.k, a.n_tok, a.k, 128, kTileM,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = make_map_2d(ctx, &mda, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.d0, a.k / QK, a.n_tok, (uint64_t)(a.k / QK) * 4,
                     kStageBlocks, kTileM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    const size_t smem = sizeof(GemmSmem) + 1024;
    static std::atomic<bool> attr[64];
    if (!attr[ctx->device & 63].load(std::memory_order_acquire)) {
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_gemm_i8, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr[ctx->device & 63].store(true, std::memory_order_release);
    }
    const dim3 grid(tiles, (p.n_tok + kTileM - 1) / kTileM);
    k_gemm_i8<<<grid, kGemmThreads, smem, ctx->stream>>>(maps, ma, mda, p);
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

static int launch_gemm_i8(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs) {
    if (sizeof(GemmSmem) + 1024 > ctx->max_smem_optin) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: smem");
    for (int i = 0; i < n_jobs; i++)
        if (!gemm_ok(a, jobs[i])) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: type or shape not supported");
    for (int i = 0; i < n_jobs; i += kMaxI8Jobs) {
        const int st = launch_i8_group(ctx, a, jobs + i, std::min(kMaxI8Jobs, n_jobs - i));
        if (st) return st;
    }
    return RCU_OK;
}

// Prefill matmul: the f16 tensor-core GEMM (every weight type) by default; the int8 GEMM with
// exact per-block sums for Q4_0 weights when the context asks for it (rcu_set_prefill_gemm).
int launch_gemm(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs) {
    if (ctx->gemm_i8) {
        bool all = true;
        for (int i = 0; i < n_jobs; i++) all &= gemm_ok(a, jobs[i]);
        if (all) return launch_gemm_i8(ctx, a, jobs, n_jobs);
    }
    return launch_gemm_f16(ctx, a, jobs, n_jobs);
}

}  // namespace rcu
