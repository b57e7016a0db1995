// rcu_quant.cu -- on-the-fly activation quantizers (Q8_0 and Q8_K) into the SoA layout
// of rcu::ActsView. Bit-exact with the reference:
//   Q8_0 scalar tier   crates/rie-core/src/quant/mod.rs:175-189   (RCU_ROUND_HALF_AWAY)
//   Q8_0 AVX2 tier     crates/rie-core/src/kernels/avx2.rs:153-184 (RCU_ROUND_NEAREST_EVEN)
//   Q8_K               crates/rie-core/src/quant/mod.rs:191-218
// Every float operation is the IEEE-rounded one the reference performs (no contraction:
// explicit __fmul_rn, IEEE division), so codes and scales match bit for bit.
#include "rcu_kernels.h"

namespace rcu {

// One warp per 32-value block, one value per lane.
__global__ void __launch_bounds__(256) k_quantize_q8_0(const float *__restrict__ x, uint32_t n_tok, uint32_t k,
                                                       int rounding, int8_t *__restrict__ q, float *__restrict__ d_out,
                                                       float *__restrict__ s_out, int32_t *__restrict__ sum_out) {
    const uint32_t nb = k / QK;
    const uint64_t blk = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (blk >= (uint64_t)n_tok * nb) return;
    const uint32_t lane = threadIdx.x & 31;
    const float v = x[blk * QK + lane];
    const float av = fabsf(v);
    // |v| >= 0, so the IEEE bit pattern orders like the value.
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(av)));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const float p = __fmul_rn(v, id);
    int r;
    if (rounding == RCU_ROUND_HALF_AWAY)
        r = __float2int_rz(roundf(p));  // f32::round then `as i32` (saturating)
    else
        r = __float2int_rn(p);  // _mm256_cvtps_epi32 with the default MXCSR
    const int c = max(-127, min(127, r));
    q[blk * QK + lane] = (int8_t)c;
    const int csum = __reduce_add_sync(0xffffffffu, c);
    const int rsum = rounding == RCU_ROUND_HALF_AWAY ? csum : __reduce_add_sync(0xffffffffu, r);
    if (lane == 0) {
        d_out[blk] = d;
        s_out[blk] = __fmul_rn(d, (float)rsum);
        sum_out[blk] = csum;
    }
}

// One CTA of 256 threads per 256-value block.
__global__ void __launch_bounds__(256) k_quantize_q8_k(const float *__restrict__ x, uint32_t n_tok, uint32_t k,
                                                       int8_t *__restrict__ q, float *__restrict__ d_out,
                                                       int16_t *__restrict__ bs_out) {
    const uint64_t blk = blockIdx.x;
    const uint32_t j = threadIdx.x, lane = j & 31, warp = j >> 5;
    const float v = x[blk * QK_K + j];
    // signed value of largest magnitude; ties keep the first index (strict > scan)
    uint64_t key = ((uint64_t)__float_as_uint(fabsf(v)) << 32) | (uint32_t)(0xffffffffu - j);
    for (int o = 16; o; o >>= 1) {
        const uint64_t other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    __shared__ uint64_t wkey[8];
    __shared__ float s_max;
    __shared__ int s_sum[16];
    if (lane == 0) wkey[warp] = key;
    __syncthreads();
    if (j == 0) {
        uint64_t best = wkey[0];
        for (int w = 1; w < 8; w++) best = wkey[w] > best ? wkey[w] : best;
        const uint32_t idx = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
        s_max = x[blk * QK_K + idx];
    }
    __syncthreads();
    const float mx = s_max;
    const bool zero = (__float_as_uint(mx) & 0x7fffffffu) == 0;
    int c = 0;
    if (!zero) {
        const float iscale = -127.0f / mx;
        c = max(-127, min(127, __float2int_rz(roundf(__fmul_rn(iscale, v)))));
        if (j == 0) d_out[blk] = 1.0f / iscale;
    } else if (j == 0) {
        d_out[blk] = 0.0f;
    }
    q[blk * QK_K + j] = (int8_t)c;
    // 16-value group sums: a group is half a warp
    int g = c;
    for (int o = 8; o; o >>= 1) g += __shfl_xor_sync(0xffffffffu, g, o);
    if ((j & 15) == 0) s_sum[j >> 4] = g;
    __syncthreads();
    if (j < 16) bs_out[blk * 16 + j] = (int16_t)s_sum[j];
}

int launch_quantize(rcu_ctx *ctx, const ActsView &a, const float *x, uint32_t n_tok, uint32_t k, uint32_t formats) {
    if (formats & RCU_ACT_Q8_0) {
        const uint64_t nblk = (uint64_t)n_tok * (k / QK);
        const uint32_t grid = (uint32_t)((nblk + 7) / 8);
        k_quantize_q8_0<<<grid, 256, 0, ctx->stream>>>(x, n_tok, k, ctx->rounding, a.q0, a.d0, a.s0, a.sum0);
        RCU_CUDA_TRY(ctx, cudaGetLastError());
    }
    if (formats & RCU_ACT_Q8K) {
        const uint64_t nblk = (uint64_t)n_tok * (k / QK_K);
        k_quantize_q8_k<<<(uint32_t)nblk, 256, 0, ctx->stream>>>(x, n_tok, k, a.qk, a.dk, a.bsk);
        RCU_CUDA_TRY(ctx, cudaGetLastError());
    }
    return RCU_OK;
}

}  // namespace rcu
