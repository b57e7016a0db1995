// rcu_gemm.cu -- prefill GEMM (n_tok > 8) on the 5th-generation tensor cores.
//
// Y[t][n] = sum_b d_a[t][b] * d_w[n][b] * S_b[t][n], with S_b the exact int32 dot of block b
// (the reference forms the same per-block ints one row at a time:
// crates/rie-core/src/kernels/matmul.rs:178-241 via vec_dot / vec_dot_x4,
// crates/rie-core/src/quant/reference.rs:221-293).
//
// Per CTA: a 128-weight-row x 128-token output tile.
//   * warp 0   TMA producer: raw GGUF weight bytes (2-D tensor map over [rows][row_bytes],
//              8 blocks = K 256 per stage), int8 activation codes (128B-swizzled, K-major)
//              and the activation block scales;
//   * warps 1-4 unpack: GGUF blocks -> int8 weight tile in the canonical 128B-swizzled
//              K-major layout the tensor core reads, plus per-row f32 block scales;
//   * warp 5   MMA issuer: one tcgen05.mma.kind::i8 (M=128, N=128, K=32) per 32-value
//              block into one of two TMEM accumulators (double buffered);
//   * warps 6-13 epilogue: tcgen05.ld the block's int32 sums, re-arm the accumulator with
//              the f32 magic 1.5*2^23 (so the next block's int sum S reads back as the
//              float 1.5*2^23 + S exactly), and fold each block into f32 accumulators with
//              two packed FMAs: t = fma(X, d_w, -1.5*2^23*d_w) = round(S * d_w) exactly
//              once, acc = fma(t, d_a, acc).
// All waits are bounded; TMEM is freed on every exit path.
#include <cuda.h>

#include <algorithm>

#include "rcu_kernels.h"
#include "rcu_tc.cuh"

namespace rcu {

constexpr int kTileN = 128;   // weight rows per CTA (MMA M)
constexpr int kTileM = 128;   // tokens per CTA (MMA N)
constexpr int kStageBlocks = 8;  // 32-value blocks per stage (K = 256)
constexpr int kStages = 2;
constexpr int kGemmThreads = 14 * 32;
constexpr uint32_t kGemmMinTok = 32;  // below this the 8-token GEMV slices are faster
constexpr uint32_t kMagicBits = 0x4B400000u;  // 1.5 * 2^23
constexpr float kMagic = 12582912.0f;

struct GemmSmem {
    // 1024-aligned operand tiles first
    uint8_t a[kStages][2][kTileN * 128];   // unpacked weights, 2 swizzle atoms of K 128
    uint8_t b[kStages][2][kTileM * 128];   // activation codes (TMA, 128B swizzle)
    uint8_t raw[kStages][kTileN * 144];    // raw GGUF bytes, 8 Q4_0 blocks (or 4.x Q8_0) per row
    float da[kStages][kTileM][kStageBlocks];
    float dw[kStages][kStageBlocks][kTileN];
    float nm[kStages][kStageBlocks][kTileN];
    uint64_t full[kStages], unpacked[kStages], empty[kStages];
    uint64_t tfull[2], tempty[2];
    uint32_t tmem_base;
};

struct GemmParams {
    const uint8_t *w;          // unused by the kernel (tensor map), kept for bounds
    float *out;
    uint64_t ld;
    uint32_t rows, k, n_tok, type, row_bytes, raw_box;  // raw_box: bytes per row per stage
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

// Unpack one 32-value block into 32 int8 codes (two 16-byte chunks, element order).
template <int TYPE>
__device__ __forceinline__ void unpack_block(const uint8_t *raw, uint32_t off, uint4 &c0, uint4 &c1, float &d) {
    if (TYPE == T_Q4_0) {
        uint32_t w[5];
        {
            const uint32_t *p = reinterpret_cast<const uint32_t *>(raw + (off & ~3u));
            const uint32_t sh = (off & 3u) * 8u;
            uint32_t r[6];
#pragma unroll
            for (int i = 0; i < 6; i++) r[i] = p[i];
#pragma unroll
            for (int i = 0; i < 5; i++) w[i] = __funnelshift_rc(r[i], r[i + 1], sh);
        }
        d = f16_bits_to_f32(w[0]);
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t q = __funnelshift_r(w[i], w[i + 1], 16);
            // nibble -> int8 (nib - 8): flip bit 3 then sign-extend the 4-bit value
            const uint32_t l = (q & 0x0F0F0F0Fu) ^ 0x08080808u, h = ((q >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
            lo[i] = l | ((l & 0x08080808u) * 30u);
            hi[i] = h | ((h & 0x08080808u) * 30u);
        }
        c0 = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        c1 = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    } else {  // Q8_0: 34-byte blocks, codes already int8
        uint32_t w[9];
        const uint32_t *p = reinterpret_cast<const uint32_t *>(raw + (off & ~3u));
        const uint32_t sh = (off & 3u) * 8u;
        uint32_t r[10];
#pragma unroll
        for (int i = 0; i < 10; i++) r[i] = p[i];
#pragma unroll
        for (int i = 0; i < 9; i++) w[i] = __funnelshift_rc(r[i], r[i + 1], sh);
        d = f16_bits_to_f32(w[0]);
        uint32_t q[8];
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = __funnelshift_r(w[i], w[i + 1], 16);
        c0 = make_uint4(q[0], q[1], q[2], q[3]);
        c1 = make_uint4(q[4], q[5], q[6], q[7]);
    }
}

template <int TYPE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_a,
           const __grid_constant__ CUtensorMap map_da, const __grid_constant__ GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    GemmSmem &S = *reinterpret_cast<GemmSmem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    constexpr uint32_t BB = TYPE == T_Q4_0 ? 18 : 34;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n0 = blockIdx.x * kTileN, m0 = blockIdx.y * kTileM;
    const uint32_t nb = p.k / QK, n_iter = nb / kStageBlocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.unpacked[s], 4);
            mbar_init(&S.empty[s], 1 + 8);  // MMA commit + 8 epilogue warps
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&S.tfull[b], 1);
            mbar_init(&S.tempty[b], 8);
        }
        fence_mbar_init();
    }
    if (warp == 5) {  // TMEM: 2 accumulators x 128 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(&S.tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;

    if (warp >= 6) {  // arm both accumulators with the magic offset
        const int e = warp - 6, q = warp & 3, h = e >> 2;
        for (int b = 0; b < 2; b++)
            for (int c = 0; c < 2; c++)
                tmem_st32_const(tmem + ((uint32_t)(32 * q) << 16) + b * 128 + 64 * h + 32 * c, kMagicBits);
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 0) {  // ---- TMA producer ----
        if (lane == 0) {
            for (uint32_t it = 0; it < n_iter; it++) {
                const uint32_t s = it % kStages;
                if (it >= kStages && !mbar_wait_bounded(&S.empty[s], ((it / kStages) - 1) & 1, p.err, ERR_TIMEOUT_EMPTY))
                    break;
                const uint32_t bytes = kTileN * p.raw_box + 2 * kTileM * 128 + kTileM * kStageBlocks * 4;
                mbar_arrive_expect_tx(&S.full[s], bytes);
                tma_load_2d(S.raw[s], &map_w, (int)(it * kStageBlocks * BB), (int)n0, &S.full[s]);
                tma_load_2d(S.b[s][0], &map_a, (int)(it * 256), (int)m0, &S.full[s]);
                tma_load_2d(S.b[s][1], &map_a, (int)(it * 256 + 128), (int)m0, &S.full[s]);
                tma_load_2d(S.da[s], &map_da, (int)(it * kStageBlocks), (int)m0, &S.full[s]);
            }
        }
    } else if (warp <= 4) {  // ---- unpack (128 threads, one weight row each) ----
        const uint32_t r = threadIdx.x - 32;
        for (uint32_t it = 0; it < n_iter; it++) {
            const uint32_t s = it % kStages;
            if (!mbar_wait_bounded(&S.full[s], (it / kStages) & 1, p.err, ERR_TIMEOUT_FULL)) break;
            const uint8_t *raw = S.raw[s] + r * p.raw_box;
#pragma unroll 2
            for (int j = 0; j < kStageBlocks; j++) {
                uint4 c0, c1;
                float d;
                unpack_block<TYPE>(raw, j * BB, c0, c1, d);
                uint8_t *rowp = S.a[s][j >> 2] + r * 128;
                const uint32_t ch = 2 * (j & 3);
                *reinterpret_cast<uint4 *>(rowp + (((ch) ^ (r & 7)) << 4)) = c0;
                *reinterpret_cast<uint4 *>(rowp + (((ch + 1) ^ (r & 7)) << 4)) = c1;
                S.dw[s][j][r] = d;
                S.nm[s][j][r] = -kMagic * d;
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.unpacked[s]);
        }
    } else if (warp == 5) {  // ---- MMA issuer ----
        if (lane == 0) {
            uint32_t b = 0;
            bool ok = true;
            for (uint32_t it = 0; it < n_iter && ok; it++) {
                const uint32_t s = it % kStages;
                if (!mbar_wait_bounded(&S.unpacked[s], (it / kStages) & 1, p.err, ERR_TIMEOUT_FULL) ||
                    !mbar_wait_bounded(&S.full[s], (it / kStages) & 1, p.err, ERR_TIMEOUT_FULL)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int j = 0; j < kStageBlocks; j++, b++) {
                    const uint32_t buf = b & 1;
                    if (!mbar_wait_bounded(&S.tempty[buf], ((b >> 1) + 1) & 1, p.err, ERR_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = sw128_desc(S.a[s][j >> 2] + 32 * (j & 3));
                    const uint64_t bd = sw128_desc(S.b[s][j >> 2] + 32 * (j & 3));
                    mma_i8(tmem + buf * 128, ad, bd);
                    mma_commit(&S.tfull[buf]);
                }
                mma_commit(&S.empty[s]);
            }
        }
    } else {  // ---- epilogue (warps 6..13) ----
        const int e = warp - 6, q = warp & 3, h = e >> 2;
        const uint32_t nrow = 32 * q + lane;  // weight row within the tile
        float2 acc[32];
#pragma unroll
        for (int c = 0; c < 32; c++) acc[c] = make_float2(0.0f, 0.0f);
        uint32_t b = 0;
        bool ok = true;
        for (uint32_t it = 0; it < n_iter && ok; it++) {
            const uint32_t s = it % kStages;
            // scales of this stage: d_a landed by TMA (full), d_w written by the unpack warps
            if (!mbar_wait_bounded(&S.full[s], (it / kStages) & 1, p.err, ERR_TIMEOUT_FULL) ||
                !mbar_wait_bounded(&S.unpacked[s], (it / kStages) & 1, p.err, ERR_TIMEOUT_FULL))
                break;
            for (int j = 0; j < kStageBlocks; j++, b++) {
                const uint32_t buf = b & 1;
                if (!mbar_wait_bounded(&S.tfull[buf], (b >> 1) & 1, p.err, ERR_TIMEOUT_FULL)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + buf * 128 + 64 * h;
                const float dw = S.dw[s][j][nrow], nm = S.nm[s][j][nrow];
                const float2 dw2 = make_float2(dw, dw), nm2 = make_float2(nm, nm);
                const float *dap = &S.da[s][64 * h][j];
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    uint32_t x[32];
                    tmem_ld32(ta + 32 * half, x);
                    tmem_wait_ld();
                    tmem_st32_const(ta + 32 * half, kMagicBits);  // re-arm for the block after next
                    if (half == 1) {
                        tmem_wait_st();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&S.tempty[buf]);
                    }
#pragma unroll
                    for (int c = 0; c < 16; c++) {
                        const int col = 32 * half + 2 * c;
                        const float2 xv = make_float2(__uint_as_float(x[2 * c]), __uint_as_float(x[2 * c + 1]));
                        const float2 da = make_float2(dap[col * kStageBlocks], dap[(col + 1) * kStageBlocks]);
                        acc[16 * half + c] = ffma2(ffma2(xv, dw2, nm2), da, acc[16 * half + c]);
                    }
                }
            }
            __syncwarp();
            if (ok && lane == 0) mbar_arrive(&S.empty[s]);
        }
        const uint32_t n = n0 + nrow;
        if (n < p.rows) {
#pragma unroll
            for (int c = 0; c < 32; c++) {
                const uint32_t m = m0 + 64 * h + 2 * c;
                if (m < p.n_tok) p.out[(uint64_t)m * p.ld + n] = acc[c].x;
                if (m + 1 < p.n_tok) p.out[(uint64_t)(m + 1) * p.ld + n] = acc[c].y;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem) : "memory");
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

template <int TYPE>
static int launch_type(rcu_ctx *ctx, const ActsView &a, const HostJob &j) {
    const rcu_weight *w = j.w;
    constexpr uint32_t BB = TYPE == T_Q4_0 ? 18 : 34;
    GemmParams p{};
    p.out = j.out;
    p.ld = j.ld;
    p.rows = (uint32_t)w->rows;
    p.k = a.k;
    p.n_tok = a.n_tok;
    p.type = TYPE;
    p.row_bytes = (uint32_t)w->row_bytes;
    p.raw_box = kStageBlocks * BB;  // 144 (Q4_0) or 272 (Q8_0) bytes per row per stage
    p.err = ctx->dev_err;
    CUtensorMap mw, ma, mda;
    int st = make_map_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->data, w->row_bytes, w->rows, w->row_bytes,
                         p.raw_box, kTileN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = make_map_2d(ctx, &ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.q0, a.k, a.n_tok, a.k, 128, kTileM,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = make_map_2d(ctx, &mda, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.d0, a.k / QK, a.n_tok, (uint64_t)(a.k / QK) * 4,
                     kStageBlocks, kTileM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    const size_t smem = sizeof(GemmSmem) + 1024;
    static bool attr[64] = {};
    if (!attr[ctx->device & 63]) {
        RCU_CUDA_TRY(ctx, cudaFuncSetAttribute(k_gemm<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr[ctx->device & 63] = true;
    }
    dim3 grid((p.rows + kTileN - 1) / kTileN, (p.n_tok + kTileM - 1) / kTileM);
    k_gemm<TYPE><<<grid, kGemmThreads, smem, ctx->stream>>>(mw, ma, mda, p);
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

static bool gemm_ok(const ActsView &a, const HostJob &j) {
    const rcu_weight *w = j.w;
    if (w->type != T_Q4_0) return false;  // other types run the GEMV in 8-token slices
    if (a.k % 256 != 0 || (w->row_bytes & 15) != 0 || (((uintptr_t)w->data) & 15) != 0) return false;
    return a.n_tok >= kGemmMinTok;
}

static int launch_gemm_i8(rcu_ctx *ctx, const ActsView &a, const HostJob *jobs, int n_jobs) {
    if (sizeof(GemmSmem) + 1024 > ctx->max_smem_optin) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: smem");
    for (int i = 0; i < n_jobs; i++)
        if (!gemm_ok(a, jobs[i])) return set_err(ctx, RCU_ERR_UNSUPPORTED, "gemm: type or shape not supported");
    for (int i = 0; i < n_jobs; i++) {
        const int st = launch_type<T_Q4_0>(ctx, a, jobs[i]);
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
