// rcu_actq.cuh -- activation quantizers as device building blocks, one value per thread.
//
// The standalone quantize kernels (rcu_quant.cu) and every kernel that produces a matmul input
// in the forward pass (norm, attention combine, GLU) call these, so there is exactly one
// implementation of the reference's rounding rules:
//   Q8_0 scalar tier   crates/rie-core/src/quant/mod.rs:175-189   (RCU_ROUND_HALF_AWAY)
//   Q8_0 AVX2 tier     crates/rie-core/src/kernels/avx2.rs:153-184 (RCU_ROUND_NEAREST_EVEN)
//   Q8_K               crates/rie-core/src/quant/mod.rs:191-218
// Every float operation is the IEEE-rounded one the reference performs (explicit __fmul_rn,
// IEEE division), so codes and scales match bit for bit.
#pragma once
#include "rcu_internal.cuh"

namespace rcu {

// Destination of a quantization: the SoA arrays of an ActsView and the formats to write.
struct ActOut {
    int8_t *q0;
    float *d0, *s0;
    int32_t *sum0;
    int8_t *qk;
    float *dk;
    int16_t *bsk;
    uint32_t fmt;
    int rounding;
};

__host__ __device__ inline ActOut act_out(const ActsView &a, uint32_t fmt, int rounding) {
    return ActOut{a.q0, a.d0, a.s0, a.sum0, a.qk, a.dk, a.bsk, fmt, rounding};
}

// The rounding step of the Q8_0 quantizer for one value: r before the clamp.
__device__ __forceinline__ int q8_0_round(float v, float id, int rounding) {
    const float p = __fmul_rn(v, id);
    if (rounding == RCU_ROUND_HALF_AWAY) return __float2int_rz(roundf(p));  // f32::round then `as i32`
    return __float2int_rn(p);  // _mm256_cvtps_epi32 with the default MXCSR
}
// The code of one value of a Q8_K block with the block's iscale = -127 / (signed max).
__device__ __forceinline__ int q8_k_code(float v, float iscale) {
    return max(-127, min(127, __float2int_rz(roundf(__fmul_rn(iscale, v)))));
}

// Q8_0 of one 32-value block held one value per lane. Called by all 32 lanes; `blk` is the
// block's index in the [token][k/32] array.
__device__ __forceinline__ void q8_0_block(float v, uint64_t blk, int lane, const ActOut &o) {
    const float av = fabsf(v);
    // |v| >= 0, so the IEEE bit pattern orders like the value.
    const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(av)));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const int r = q8_0_round(v, id, o.rounding);
    const int c = max(-127, min(127, r));
    o.q0[blk * QK + lane] = (int8_t)c;
    const int csum = __reduce_add_sync(0xffffffffu, c);
    const int rsum = o.rounding == RCU_ROUND_HALF_AWAY ? csum : __reduce_add_sync(0xffffffffu, r);
    if (lane == 0) {
        o.d0[blk] = d;
        o.s0[blk] = __fmul_rn(d, (float)rsum);
        o.sum0[blk] = csum;
    }
}

// Scratch for q8_k_block: one key and value per warp of the CTA, two copies so that back to
// back calls need only the one __syncthreads inside.
struct Q8kShared {
    unsigned long long key[2][32];
    float val[2][32];
};

// Q8_K of one 256-value block held one value per thread by 8 consecutive warps
// (j = index in the block, 0..255; the block's first warp is warp `w0` of the CTA).
// Every participating thread must call this the same number of times: it synchronises the
// whole CTA (bar_threads == 0) or the first bar_threads threads on named barrier bar_id.
// `store` false skips the writes (threads past the end of the row). `parity` alternates.
__device__ __forceinline__ void q8_k_block(float v, uint32_t j, uint32_t w0, uint64_t blk, bool store,
                                           const ActOut &o, Q8kShared &sh, int parity, int bar_id = 0,
                                           int bar_threads = 0) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // signed value of largest magnitude; ties keep the first index (strict > scan)
    unsigned long long key = ((unsigned long long)__float_as_uint(fabsf(v)) << 32) | (uint32_t)(0xffffffffu - j);
    for (int off = 16; off; off >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, off);
        key = other > key ? other : key;
    }
    const float wv = __shfl_sync(0xffffffffu, v, (int)((0xffffffffu - (uint32_t)(key & 0xffffffffu)) & 31));
    if (lane == 0) {
        sh.key[parity][warp] = key;
        sh.val[parity][warp] = wv;
    }
    if (bar_threads)
        asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(bar_threads) : "memory");
    else
        __syncthreads();
    unsigned long long best = sh.key[parity][w0];
    float mx = sh.val[parity][w0];
#pragma unroll
    for (uint32_t w = 1; w < 8; w++) {
        const unsigned long long k2 = sh.key[parity][w0 + w];
        if (k2 > best) {
            best = k2;
            mx = sh.val[parity][w0 + w];
        }
    }
    const bool zero = (__float_as_uint(mx) & 0x7fffffffu) == 0;
    int c = 0;
    float d = 0.0f;
    if (!zero) {
        const float iscale = -127.0f / mx;
        c = q8_k_code(v, iscale);
        d = 1.0f / iscale;
    }
    // 16-value group sums: a group is half a warp
    int g = c;
    for (int off = 8; off; off >>= 1) g += __shfl_xor_sync(0xffffffffu, g, off);
    if (store) {
        o.qk[blk * QK_K + j] = (int8_t)c;
        if (j == 0) o.dk[blk] = d;
        if ((j & 15) == 0) o.bsk[blk * 16 + (j >> 4)] = (int16_t)g;
    }
}

// ---- eight consecutive values per lane ------------------------------------------------------
// The same quantizers for kernels whose lanes hold 8 consecutive values of a row (two float4
// loads): a Q8_0 block is 4 lanes (lane & ~3 .. +3), a Q8_K block a whole warp, so neither
// needs shared memory or a CTA barrier. Every lane of the warp calls them; `store` false skips
// the writes of lanes past the row's end (Q8_0 only: the row holds whole 32-value blocks).

__device__ __forceinline__ uint32_t pack_codes4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) | ((uint32_t)d << 24);
}

// blk: index of this quad's block in the [token][k/32] array; values 8 (lane & 3) .. +7 of it.
__device__ __forceinline__ void q8_0_block8(const float (&v)[8], uint64_t blk, uint32_t lane, bool store,
                                            const ActOut &o) {
    uint32_t am = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) am = max(am, __float_as_uint(fabsf(v[i])));
    am = max(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = max(am, __shfl_xor_sync(0xffffffffu, am, 2));
    const float d = __uint_as_float(am) / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    int c[8], csum = 0, rsum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = q8_0_round(v[i], id, o.rounding);
        c[i] = max(-127, min(127, r));
        csum += c[i];
        rsum += r;
    }
    csum += __shfl_xor_sync(0xffffffffu, csum, 1);
    csum += __shfl_xor_sync(0xffffffffu, csum, 2);
    rsum += __shfl_xor_sync(0xffffffffu, rsum, 1);
    rsum += __shfl_xor_sync(0xffffffffu, rsum, 2);
    if (!store) return;
    *reinterpret_cast<uint2 *>(o.q0 + blk * QK + 8 * (lane & 3)) =
        make_uint2(pack_codes4(c[0], c[1], c[2], c[3]), pack_codes4(c[4], c[5], c[6], c[7]));
    if ((lane & 3) == 0) {
        o.d0[blk] = d;
        o.s0[blk] = __fmul_rn(d, (float)(o.rounding == RCU_ROUND_HALF_AWAY ? csum : rsum));
        o.sum0[blk] = csum;
    }
}

// blk: index of the warp's block in the [token][k/256] array; values 8 lane .. 8 lane + 7.
__device__ __forceinline__ void q8_k_block8(const float (&v)[8], uint64_t blk, uint32_t lane, const ActOut &o) {
    // signed value of largest magnitude; ties keep the first index (strict > scan)
    unsigned long long key = 0;
    float best = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const unsigned long long k2 =
            ((unsigned long long)__float_as_uint(fabsf(v[i])) << 32) | (uint32_t)(0xffffffffu - (8 * lane + i));
        if (k2 > key) key = k2, best = v[i];
    }
    for (int off = 16; off; off >>= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, off);
        const float b2 = __shfl_xor_sync(0xffffffffu, best, off);
        if (k2 > key) key = k2, best = b2;
    }
    const bool zero = (__float_as_uint(best) & 0x7fffffffu) == 0;
    const float iscale = zero ? 0.0f : -127.0f / best;
    int c[8], g = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        c[i] = zero ? 0 : q8_k_code(v[i], iscale);
        g += c[i];
    }
    g += __shfl_xor_sync(0xffffffffu, g, 1);  // 16-value group = lane pair
    *reinterpret_cast<uint2 *>(o.qk + blk * QK_K + 8 * lane) =
        make_uint2(pack_codes4(c[0], c[1], c[2], c[3]), pack_codes4(c[4], c[5], c[6], c[7]));
    if ((lane & 1) == 0) o.bsk[blk * 16 + lane / 2] = (int16_t)g;
    if (lane == 0) o.dk[blk] = zero ? 0.0f : 1.0f / iscale;
}

}  // namespace rcu
