// rcu_wquant.cu -- weight quantization on the device: f32 rows -> GGUF blocks.
//
//   Q8_0, Q4_0      the reference's weight quantizers (crates/rie-core/src/quant/mod.rs:262-307)
//   Q4_1, Q5_0, Q5_1, Q4_K, Q5_K, Q6_K
//                   this library's own rules: the reference has no quantizer for these types
//                   (its models arrive quantized), so they are restated from the block layouts
//                   of quant/reference.rs:53-207 (min/max per 32-value sub-block, 6-bit scale /
//                   min codes against one f16 scale per superblock; Q6_K: 16 signed 8-bit group
//                   scales, q + 32 in 6 bits). Valid blocks, not tuned for error.
//
// Used to build models from f32 weights on the GPU (the benchmark configurations draw their
// weights from N(0, 0.02) and quantize them). One thread per block; every float operation is
// written out with explicit rounding (no contraction into fused multiply-adds), so the bytes
// equal the CPU restatement's bit for bit.
#include <algorithm>

#include "rcu_kernels.h"

namespace rcu {
namespace {

// The f16 fields sit at even offsets of the (2-byte aligned) block: one 16-bit store.
__device__ __forceinline__ void put_f16(uint8_t *p, float v) {
    *reinterpret_cast<uint16_t *>(p) = __half_as_ushort(__float2half_rn(v));
}
__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
// Rust `f32 as i32` (saturating, NaN -> 0): the PTX conversion with truncation does exactly that.
__device__ __forceinline__ int sat_i32(float v) { return __float2int_rz(v); }

// Q4_K / Q5_K scale and min codes of 8 sub-blocks into the 12 packed bytes (the inverse of
// get_scale_min_k4, reference.rs:8-14).
__device__ __forceinline__ void k4_pack(const uint8_t (&sc)[8], const uint8_t (&mn)[8], uint8_t *q) {
    uint8_t b[12] = {};
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            b[j] |= sc[j] & 63;
            b[j + 4] |= mn[j] & 63;
        } else {
            b[j + 4] |= (uint8_t)((sc[j] & 0xF) | ((mn[j] & 0xF) << 4));
            b[j - 4] |= (uint8_t)((sc[j] >> 4) << 6);
            b[j] |= (uint8_t)((mn[j] >> 4) << 6);
        }
    }
#pragma unroll
    for (int j = 0; j < 12; j++) q[j] = b[j];
}

template <int T>
__device__ void quantize_block(const float *x, uint8_t *o) {
    if (T == T_Q8_0) {  // quant/mod.rs:265-277
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
        const float d = __fdiv_rn(amax, 127.0f), id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        put_f16(o, d);
        for (int j = 0; j < 32; j++) o[2 + j] = (uint8_t)(int8_t)clampi(sat_i32(roundf(__fmul_rn(x[j], id))), -127, 127);
    } else if (T == T_Q4_0 || T == T_Q5_0) {  // quant/mod.rs:279-298 (Q5_0: the same rule with 5 bits)
        float mx = 0.0f;
        for (int j = 0; j < 32; j++)
            if (fabsf(x[j]) > fabsf(mx)) mx = x[j];
        const float d = __fdiv_rn(mx, T == T_Q4_0 ? -8.0f : -16.0f), id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float off = T == T_Q4_0 ? 8.5f : 16.5f;
        const int top = T == T_Q4_0 ? 15 : 31;
        put_f16(o, d);
        uint32_t qh = 0;
        for (int j = 0; j < 16; j++) {
            const int q0 = clampi(sat_i32(__fadd_rn(__fmul_rn(x[j], id), off)), 0, top);
            const int q1 = clampi(sat_i32(__fadd_rn(__fmul_rn(x[j + 16], id), off)), 0, top);
            if (T == T_Q4_0) {
                o[2 + j] = (uint8_t)(q0 | (q1 << 4));
            } else {
                o[6 + j] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
                qh |= (uint32_t)(q0 >> 4) << j;
                qh |= (uint32_t)(q1 >> 4) << (j + 16);
            }
        }
        if (T == T_Q5_0)
            for (int i = 0; i < 4; i++) o[2 + i] = (uint8_t)(qh >> (8 * i));
    } else if (T == T_Q4_1 || T == T_Q5_1) {
        const int nq = T == T_Q4_1 ? 15 : 31;
        float mn = x[0], mx = x[0];
        for (int j = 1; j < 32; j++) mn = fminf(mn, x[j]), mx = fmaxf(mx, x[j]);
        const float d = __fdiv_rn(__fsub_rn(mx, mn), (float)nq), id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        put_f16(o, d);
        put_f16(o + 2, mn);
        uint8_t q[32];
        for (int j = 0; j < 32; j++)
            q[j] = (uint8_t)clampi(__float2int_rz(__fadd_rn(__fmul_rn(__fsub_rn(x[j], mn), id), 0.5f)), 0, nq);
        if (T == T_Q4_1) {
            for (int j = 0; j < 16; j++) o[4 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
        } else {
            uint32_t qh = 0;
            for (int j = 0; j < 16; j++) {
                o[8 + j] = (uint8_t)((q[j] & 0xF) | ((q[j + 16] & 0xF) << 4));
                qh |= (uint32_t)((q[j] >> 4) & 1) << j;
                qh |= (uint32_t)((q[j + 16] >> 4) & 1) << (j + 16);
            }
            for (int i = 0; i < 4; i++) o[4 + i] = (uint8_t)(qh >> (8 * i));
        }
    } else if (T == T_Q4_K || T == T_Q5_K) {
        const int nq = T == T_Q4_K ? 15 : 31;
        float scale[8], mins[8];
        for (int j = 0; j < 8; j++) {
            float mn = x[32 * j], mx = x[32 * j];
            for (int l = 1; l < 32; l++) mn = fminf(mn, x[32 * j + l]), mx = fmaxf(mx, x[32 * j + l]);
            if (mn > 0.0f) mn = 0.0f;
            scale[j] = __fdiv_rn(__fsub_rn(mx, mn), (float)nq);
            mins[j] = -mn;
        }
        float ms = 0.0f, mm = 0.0f;
        for (int j = 0; j < 8; j++) ms = fmaxf(ms, scale[j]), mm = fmaxf(mm, mins[j]);
        const float d = __fdiv_rn(ms, 63.0f), dmin = __fdiv_rn(mm, 63.0f);
        put_f16(o, d);
        put_f16(o + 2, dmin);
        const float dh = f16_round(d), dmh = f16_round(dmin);
        uint8_t sc[8], mq[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = (uint8_t)clampi(dh > 0.0f ? (int)lroundf(__fdiv_rn(scale[j], dh)) : 0, 0, 63);
            mq[j] = (uint8_t)clampi(dmh > 0.0f ? (int)lroundf(__fdiv_rn(mins[j], dmh)) : 0, 0, 63);
        }
        k4_pack(sc, mq, o + 4);
        if (T == T_Q5_K)
            for (int l = 0; l < 32; l++) o[16 + l] = 0;
        for (int j = 0; j < 8; j++) {
            const float dd = __fmul_rn(dh, (float)sc[j]), m = __fmul_rn(dmh, (float)mq[j]);
            const int pair = j >> 1, hi = j & 1;  // sub-block j: low (hi = 0) / high nibbles of bytes 32 * pair + l
            for (int l = 0; l < 32; l++) {
                const int q = clampi(dd > 0.0f ? (int)lroundf(__fdiv_rn(__fadd_rn(x[32 * j + l], m), dd)) : 0, 0, nq);
                if (T == T_Q4_K) {
                    uint8_t &b = o[16 + 32 * pair + l];
                    b = hi ? (uint8_t)(b | (q << 4)) : (uint8_t)q;
                } else {
                    uint8_t &b = o[48 + 32 * pair + l];
                    b = hi ? (uint8_t)(b | ((q & 0xF) << 4)) : (uint8_t)(q & 0xF);
                    o[16 + l] |= (uint8_t)(((q >> 4) & 1) << (2 * pair + hi));
                }
            }
        }
    } else {  // Q6_K
        float sc_f[16];
        float amax_all = 0.0f;
        for (int g = 0; g < 16; g++) {
            float m = 0.0f;
            for (int l = 0; l < 16; l++) m = fmaxf(m, fabsf(x[16 * g + l]));
            sc_f[g] = __fdiv_rn(m, 31.0f);
            amax_all = fmaxf(amax_all, sc_f[g]);
        }
        const float d = __fdiv_rn(amax_all, 127.0f);
        put_f16(o + 208, d);
        const float dh = f16_round(d);
        int8_t sc[16];
        for (int g = 0; g < 16; g++) {
            sc[g] = (int8_t)clampi(dh > 0.0f ? (int)lroundf(__fdiv_rn(sc_f[g], dh)) : 0, -128, 127);
            o[192 + g] = (uint8_t)sc[g];
        }
        uint8_t *ql = o, *qh = o + 128;
        for (int i = 0; i < 128; i++) ql[i] = 0;
        for (int i = 0; i < 64; i++) qh[i] = 0;
        for (int g = 0; g < 16; g++) {
            const float dd = __fmul_rn(dh, (float)sc[g]);
            for (int l = 0; l < 16; l++) {
                const int i = 16 * g + l;  // value index within the superblock
                const uint8_t q = (uint8_t)clampi((dd != 0.0f ? (int)lroundf(__fdiv_rn(x[i], dd)) : 0) + 32, 0, 63);
                // reference.rs:190-207 layout: value i = 128 n + 32 m + c (m = 0..3, c = 0..31)
                const int n = i >> 7, m = (i >> 5) & 3, c = i & 31;
                uint8_t &lo = ql[64 * n + 32 * (m & 1) + c];
                lo = (m >> 1) ? (uint8_t)(lo | ((q & 0xF) << 4)) : (uint8_t)(lo | (q & 0xF));
                qh[32 * n + c] |= (uint8_t)((q >> 4) << (2 * m));
            }
        }
    }
}

template <int T>
__global__ void k_quantize_weight(const float *__restrict__ x, uint64_t rows, uint64_t cols, uint64_t ld,
                                  uint8_t *__restrict__ out) {
    constexpr int BS = T == T_Q4_K || T == T_Q5_K || T == T_Q6_K ? QK_K : QK;
    const uint64_t per_row = cols / BS, n = rows * per_row;
    constexpr uint32_t bb = T == T_Q4_0 ? 18 : T == T_Q4_1 ? 20 : T == T_Q5_0 ? 22 : T == T_Q5_1 ? 24 : T == T_Q8_0 ? 34
                            : T == T_Q4_K ? 144 : T == T_Q5_K ? 176 : 210;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / per_row, b = i % per_row;
        // the block is built in local memory and stored as 16-bit words (every GGUF block is a
        // whole number of them and 2-byte aligned): no byte-wise read-modify-write of the output
        uint16_t blk[bb / 2];
        quantize_block<T>(x + r * ld + b * BS, reinterpret_cast<uint8_t *>(blk));
        uint16_t *dst = reinterpret_cast<uint16_t *>(out + i * bb);
#pragma unroll
        for (uint32_t w = 0; w < bb / 2; w++) dst[w] = blk[w];
    }
}

template <int T>
int launch_wq(rcu_ctx *ctx, const float *x, uint64_t rows, uint64_t cols, uint64_t ld, uint8_t *out) {
    const uint64_t blocks = rows * cols / (uint64_t)block_size(T);
    const uint32_t grid = (uint32_t)std::min<uint64_t>((blocks + 127) / 128, (uint64_t)ctx->num_sms * 16);
    k_quantize_weight<T><<<std::max<uint32_t>(grid, 1), 128, 0, ctx->stream>>>(x, rows, cols, ld, out);
    RCU_CUDA_TRY(ctx, cudaGetLastError());
    return RCU_OK;
}

}  // namespace
}  // namespace rcu

using namespace rcu;

extern "C" {

int32_t rcu_quantize_weight(rcu_ctx *ctx, uint32_t ggml_type, uint64_t rows, uint64_t cols, const float *x_dev,
                            uint64_t ld, void *out_dev) {
    if (!ctx || !x_dev || !out_dev) return set_err(ctx, RCU_ERR_INVALID, "null argument");
    const int bs = block_size((int)ggml_type);
    if (bs <= 1 || ggml_type == T_Q2_K || ggml_type == T_Q3_K)
        return set_err(ctx, RCU_ERR_UNSUPPORTED, "quantize_weight: no quantizer for ggml type " + std::to_string(ggml_type));
    if (cols == 0 || cols % bs) return set_err(ctx, RCU_ERR_INVALID, "quantize_weight: cols not a multiple of the block size");
    if (ld < cols) return set_err(ctx, RCU_ERR_INVALID, "quantize_weight: ld smaller than cols");
    if (rows == 0) return RCU_OK;
    uint8_t *out = reinterpret_cast<uint8_t *>(out_dev);
    switch (ggml_type) {
        case T_Q4_0: return launch_wq<T_Q4_0>(ctx, x_dev, rows, cols, ld, out);
        case T_Q4_1: return launch_wq<T_Q4_1>(ctx, x_dev, rows, cols, ld, out);
        case T_Q5_0: return launch_wq<T_Q5_0>(ctx, x_dev, rows, cols, ld, out);
        case T_Q5_1: return launch_wq<T_Q5_1>(ctx, x_dev, rows, cols, ld, out);
        case T_Q8_0: return launch_wq<T_Q8_0>(ctx, x_dev, rows, cols, ld, out);
        case T_Q4_K: return launch_wq<T_Q4_K>(ctx, x_dev, rows, cols, ld, out);
        case T_Q5_K: return launch_wq<T_Q5_K>(ctx, x_dev, rows, cols, ld, out);
        default: return launch_wq<T_Q6_K>(ctx, x_dev, rows, cols, ld, out);
    }
}

}  // extern "C"
