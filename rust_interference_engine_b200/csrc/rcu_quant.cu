// rcu_quant.cu -- on-the-fly activation quantizers (Q8_0 and Q8_K) into the SoA layout
// of rcu::ActsView, bit-exact with the reference (the rounding rules live in rcu_actq.cuh).
#include "rcu_actq.cuh"
#include "rcu_kernels.h"

namespace rcu {

// One warp per 32-value block, one value per lane.
__global__ void __launch_bounds__(256) k_quantize_q8_0(const float *__restrict__ x, uint32_t n_tok, uint32_t k,
                                                       const ActOut o) {
    pdl_wait();
    pdl_trigger();
    const uint32_t nb = k / QK;
    const uint64_t blk = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (blk >= (uint64_t)n_tok * nb) return;
    const int lane = threadIdx.x & 31;
    q8_0_block(x[blk * QK + lane], blk, lane, o);
}

// One CTA of 256 threads per 256-value block.
__global__ void __launch_bounds__(256) k_quantize_q8_k(const float *__restrict__ x, const ActOut o) {
    pdl_wait();
    pdl_trigger();
    __shared__ Q8kShared sh;
    const uint64_t blk = blockIdx.x;
    q8_k_block(x[blk * QK_K + threadIdx.x], threadIdx.x, 0, blk, true, o, sh, 0);
}

// Eight consecutive values per lane (two float4 loads): a warp quantizes 256 values of the
// flat [n_tok][k] array, i.e. one Q8_K block or eight Q8_0 blocks, with no CTA barrier.
constexpr int kQuant8Threads = 256;
__global__ void __launch_bounds__(kQuant8Threads) k_quantize_v8(const float *__restrict__ x, uint64_t total,
                                                                const ActOut o) {
    pdl_wait();
    pdl_trigger();
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t i0 = ((uint64_t)blockIdx.x * kQuant8Threads + threadIdx.x) * 8;
    const bool in = i0 < total;
    float v[8];
    if (in) {
        const float4 a = reinterpret_cast<const float4 *>(x + i0)[0], b = reinterpret_cast<const float4 *>(x + i0)[1];
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = 0.0f;
    }
    if (o.fmt & RCU_ACT_Q8_0) q8_0_block8(v, i0 / QK, lane, in, o);
    if ((o.fmt & RCU_ACT_Q8K) && (i0 & ~(uint64_t)(QK_K - 1)) < total) q8_k_block8(v, i0 / QK_K, lane, o);
}

int launch_quantize(rcu_ctx *ctx, const ActsView &a, const float *x, uint32_t n_tok, uint32_t k, uint32_t formats) {
    const ActOut o = act_out(a, formats, ctx->rounding);
    if ((((uintptr_t)x) & 15) == 0) {  // aligned rows: the barrier-free kernel for both formats
        const uint64_t total = (uint64_t)n_tok * k;
        const uint64_t grid = (total + 8 * kQuant8Threads - 1) / (8 * kQuant8Threads);
        if (grid && grid < (1u << 31)) {
            RCU_CUDA_TRY(ctx, launch_k(ctx, (k_quantize_v8), dim3((uint32_t)grid), dim3(kQuant8Threads), 0, x, total, o));
            return RCU_OK;
        }
    }
    if (formats & RCU_ACT_Q8_0) {
        const uint64_t nblk = (uint64_t)n_tok * (k / QK);
        const uint32_t grid = (uint32_t)((nblk + 7) / 8);
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_quantize_q8_0), dim3(grid), dim3(256), 0, x, n_tok, k, o));
        RCU_CUDA_TRY(ctx, cudaGetLastError());
    }
    if (formats & RCU_ACT_Q8K) {
        const uint64_t nblk = (uint64_t)n_tok * (k / QK_K);
        RCU_CUDA_TRY(ctx, launch_k(ctx, (k_quantize_q8_k), dim3((uint32_t)nblk), dim3(256), 0, x, o));
        RCU_CUDA_TRY(ctx, cudaGetLastError());
    }
    return RCU_OK;
}

}  // namespace rcu
